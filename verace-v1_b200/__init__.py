"""B200-native (sm_100a) SSSD + CHAM sequence-mixing path for Verace V1 (placeholder)."""
