"""Sequence-parallel SSSD and CHAM scans for long sequences on few chains (benchmark
config 4: one sequence of 65536 tokens, 16 SSSD heads, one hologram).

The reference scans in O(log S) depth with a Blelloch prefix over the per-token factors
(sssd_attention.py:185-217, cham_memory.py:246-293); the chunked kernels of this package
walk the chunks of a chain in order, one CTA (SSSD) or D/32 CTAs (CHAM) per chain, so a
single sequence would occupy 16 or 32 of the 148 SMs.  Here the sequence is cut into R
contiguous ranges that run side by side as R independent chains:

1. range transforms: each range scanned from the identity gives its product
   P_r = U_{end(r)} ... U_{start(r)}  (the same scan kernels, batch b*R);
2. carry: the state entering range r is S_r = P_{r-1} S_{r-1}, S_0 = the caller's initial
   state: R - 1 dense products in fp32 (cuBLAS SGEMM / CGEMM through torch: plain
   library GEMMs, a few per call);
3. each range scanned again from its carried state S_r, giving every token's readout and
   the final state (the carried holograms are products of unitary factors, so the CHAM
   launcher continues them on the tensor cores after its unitarity probe).  Range 0 of a
   single sequence that starts from the identity already has its readouts from step 1, so
   step 3 then runs ranges 1..R-1 only.

Both passes fill the GPU (b*R chains), which is what turns config 4 from a walk along one
chain into work for all SMs.  The same split runs across GPUs (``group``): each rank
takes one contiguous segment of the sequence, and the segment products are exchanged with
one NCCL all_gather per mixer (8 MiB per rank for a D = 1024 hologram), so every rank can
form the state entering its own segment.  The arithmetic is the reference's: the same factors, the
same products, in another association order (as the reference's own Blelloch scan).  A
range length is a multiple of 64 tokens; the sequence is padded at its end with tokens
whose factors are the identity (k = v = 0, gate 0), whose outputs are dropped.
"""
from typing import Optional, Tuple

import torch

CHUNK = 64


def _sms(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


MIN_RANGE = 32 * CHUNK   # 2048 tokens: shorter sequences gain less than the second pass costs


def pick_ranges(chain_ctas: int, s: int, device, per_sm: int, min_range: int = MIN_RANGE) -> int:
    """Ranges to cut a sequence of s tokens into: the largest power of two R such that the
    R-fold chains (chain_ctas CTAs per chain, per_sm resident per SM) still run in one wave
    and every range keeps at least `min_range` tokens; 1 when that is 1."""
    slots = per_sm * _sms(device)
    R = 1
    while 2 * R * chain_ctas <= slots and s >= 2 * R * min_range:
        R *= 2
    return R


def _pad(x: torch.Tensor, total: int) -> torch.Tensor:
    """x [b, s, ...] -> [b, total, ...] with zero tokens appended (a copy only if needed)."""
    b, s = x.shape[:2]
    if s == total:
        return x.contiguous()
    out = x.new_zeros((b, total) + tuple(x.shape[2:]))
    out[:, :s] = x
    return out


def _carry(P: torch.Tensor, S0: torch.Tensor) -> torch.Tensor:
    """P [b, R, ...m, m] (range products), S0 [b, ...m, m] -> the states entering each range,
    [b, R, ...m, m]: S_0 = S0, S_r = P_{r-1} S_{r-1}."""
    R = P.shape[1]
    starts = torch.empty_like(P)
    S = S0
    for r in range(R):
        starts[:, r] = S
        if r + 1 < R:
            S = torch.matmul(P[:, r], S)
    return starts


def _prior_product(T: torch.Tensor, S0: torch.Tensor, group) -> torch.Tensor:
    """Sequence-parallel ranks: T [..., m, m] is this rank's whole-segment product (its
    ranges' products chained); every rank's T is gathered (one NCCL all_gather) and the
    state entering this rank's segment, T_{rank-1} ... T_0 S0, is formed (every rank forms
    the same chain; the segments are in rank order along the sequence)."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    real = torch.view_as_real(T.contiguous()) if T.is_complex() else T.contiguous()
    allT = torch.empty((world * real.shape[0],) + tuple(real.shape[1:]), dtype=real.dtype, device=real.device)
    dist.all_gather_into_tensor(allT, real, group=group)
    allT = allT.view((world,) + tuple(real.shape))
    if T.is_complex():
        allT = torch.view_as_complex(allT)
    S = S0
    for j in range(rank):
        S = torch.matmul(allT[j], S)
    return S


def _segment_product(P: torch.Tensor) -> torch.Tensor:
    """P [b, R, ..., m, m] -> P_{R-1} ... P_0, [b, ..., m, m]."""
    T = P[:, 0]
    for r in range(1, P.shape[1]):
        T = torch.matmul(P[:, r], T)
    return T


def sssd_scan_ranges(q, k, v, delta, initial_state: Optional[torch.Tensor], R: int, group=None
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    """launch_sssd_scan's contract (q, k, v [b, s, h, d], delta [b, s, h]) computed over R
    sequence ranges (module docstring).  With a process group, the arguments are this
    rank's segment of a sequence split over the ranks in rank order, and initial_state is
    the state before the first segment (the same on every rank); the returned state is the
    one after this rank's segment."""
    from .kernels import launch_sssd_scan
    b, s, h, d = q.shape
    L = -(-s // (R * CHUNK)) * CHUNK
    n = R * L
    qp, kp, vp = (_pad(x, n).view(b * R, L, h, d) for x in (q, k, v))
    dp = _pad(delta.reshape(b, s, h).float(), n).view(b * R, L, h)
    out1, P = launch_sssd_scan(qp, kp, vp, dp, _ranges=False)         # [b*R, h, d, d]
    P = P.view(b, R, h, d, d)
    if initial_state is None:
        S0 = torch.eye(d, device=q.device, dtype=torch.float32).expand(b, h, d, d)
    else:
        S0 = initial_state.float().reshape(b, h, d, d)
    if group is not None:
        S0 = _prior_product(_segment_product(P), S0, group)
    starts = _carry(P, S0)
    if b == 1 and initial_state is None and group is None and R > 1:   # range 0's readouts are final
        out1 = out1.view(R, L, h, d)
        out, psi = launch_sssd_scan(qp[1:], kp[1:], vp[1:], dp[1:], initial_state=starts[0, 1:].contiguous(),
                                    _ranges=False)
        full = torch.cat([out1[:1], out], dim=0).view(1, n, h, d)
        return full[:, :s], psi[-1:].contiguous()
    out, psi = launch_sssd_scan(qp, kp, vp, dp, initial_state=starts.view(b * R, h, d, d), _ranges=False)
    return out.view(b, n, h, d)[:, :s], psi.view(b, R, h, d, d)[:, -1].contiguous()


def cham_scan_ranges(q, k, v, gamma, initial_hologram: Optional[Tuple[torch.Tensor, torch.Tensor]], R: int,
                     group=None) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """launch_cham_update's contract (q, k, v [b, s, D], gamma [b, s]) computed over R
    sequence ranges (module docstring); with a process group as sssd_scan_ranges."""
    from .kernels import launch_cham_update
    b, s, D = q.shape
    L = -(-s // (R * CHUNK)) * CHUNK
    n = R * L
    qp, kp, vp = (_pad(x, n).view(b * R, L, D) for x in (q, k, v))
    gp = _pad(gamma.reshape(b, s).float(), n).view(b * R, L)
    out1, (Pr, Pi) = launch_cham_update(qp, kp, vp, gp, _ranges=False)   # range products from I
    P = torch.complex(Pr, Pi).view(b, R, D, D)
    del Pr, Pi
    if initial_hologram is None:
        S0 = torch.eye(D, device=q.device, dtype=torch.complex64).expand(b, D, D)
    else:
        S0 = torch.complex(initial_hologram[0].float(), initial_hologram[1].float()).reshape(b, D, D)
    if group is not None:
        S0 = _prior_product(_segment_product(P), S0, group)
    starts = _carry(P, S0).view(b * R, D, D)
    del P
    if b == 1 and initial_hologram is None and group is None and R > 1:   # range 0's readouts are final
        st = starts[1:]
        out, (Hr, Hi) = launch_cham_update(qp[1:], kp[1:], vp[1:], gp[1:], initial_hologram=(st.real, st.imag),
                                           _ranges=False)
        full = torch.cat([out1.view(R, L, D)[:1], out], dim=0).view(1, n, D)
        return full[:, :s], (Hr[-1:].contiguous(), Hi[-1:].contiguous())
    del out1
    out, (Hr, Hi) = launch_cham_update(qp, kp, vp, gp, initial_hologram=(starts.real, starts.imag), _ranges=False)
    Hr = Hr.view(b, R, D, D)[:, -1].contiguous()
    Hi = Hi.view(b, R, D, D)[:, -1].contiguous()
    return out.view(b, n, D)[:, :s], (Hr, Hi)
