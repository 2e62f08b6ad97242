"""Host logic of the batched ACDE loop (verace_v1_b200.AdaptiveCognitiveDepthEngine), on CPU.

The reference loop (acd_engine.py:94-156) runs each layer once per batch item on that
item's gathered active tokens; the batched loop runs each layer once on the whole batch
under the active mask.  With a layer whose recurrence skips masked tokens, the two must
agree: outputs, ponder costs (N + R), and per-layer per-item states, including the
states the reference never touches (an item with no active token at a layer, layers
after every token has halted).  The layer here is a small CPU stand-in with the real
layer's call signature and a genuine recurrence over tokens; the gathered loop is
restated below from acd_engine.py.
"""
import pytest
import torch
import torch.nn as nn

import verace_v1_b200 as V


class _Dims:
    def __init__(self, **kw):
        self.__dict__.update(kw)


class RecurrentStandIn(nn.Module):
    """(h_in, block_residual, sssd_state, cham_hologram, active_mask) -> (h_out, block_residual,
    psi [b,1,2,2], (Hr [b,2,2], Hi [b,2,2])): each active token rotates the states by an
    angle from its features and reads them out; masked tokens leave the states unchanged
    (the identity factor a zero gate gives)."""

    def __init__(self, hidden, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.w = nn.Parameter(torch.randn(hidden, 2, generator=g) * 0.3, requires_grad=False)
        self.sssd_attn = _Dims(num_heads=1, head_dim=2)
        self.cham_memory = _Dims(holographic_dim=2)

    def forward(self, h_in, block_residual=None, sssd_state=None, cham_hologram=None, active_mask=None):
        b, s, d = h_in.shape
        psi = torch.eye(2).expand(b, 1, 2, 2).clone() if sssd_state is None else sssd_state.clone()
        hr, hi = ((torch.eye(2).expand(b, 2, 2).clone(), torch.zeros(b, 2, 2)) if cham_hologram is None
                  else (cham_hologram[0].clone(), cham_hologram[1].clone()))
        out = torch.empty_like(h_in)
        for t in range(s):
            a = h_in[:, t] @ self.w                                   # [b, 2]
            c, sn = torch.cos(a[:, 0]), torch.sin(a[:, 0])
            rot = torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)   # [b, 2, 2]
            act = torch.ones(b, dtype=torch.bool) if active_mask is None else active_mask[:, t]
            new_psi = rot.unsqueeze(1) @ psi
            new_hr = rot @ hr + 0.1 * a[:, 1, None, None] * hi
            new_hi = rot @ hi - 0.1 * a[:, 1, None, None] * hr
            psi = torch.where(act[:, None, None, None], new_psi, psi)
            hr = torch.where(act[:, None, None], new_hr, hr)
            hi = torch.where(act[:, None, None], new_hi, hi)
            read = torch.cat([psi.reshape(b, 4), hr.reshape(b, 4)], -1)  # [b, 8]
            out[:, t] = torch.tanh(h_in[:, t] + read.repeat(1, d // 8))
        return out, block_residual, psi, (hr, hi)


def gathered_reference_loop(acde, layers, h_in, max_depth, min_depth, initial_layer_states=None):
    """acd_engine.py:36-167 restated: per layer, per item, the item's active tokens only."""
    b, s, d = h_in.shape
    h_curr = h_in.clone()
    final_h = torch.zeros_like(h_in)
    acc = torch.zeros(b, s)
    depth = torch.zeros(b, s)
    active = torch.ones(b, s, dtype=torch.bool)
    nl = min(len(layers), max_depth)
    states = [(list(initial_layer_states[l]) if initial_layer_states is not None and l < len(initial_layer_states)
               and initial_layer_states[l] is not None else [None] * b) for l in range(nl)]
    for l in range(nl):
        if not active.any():
            break
        h_next = h_curr.clone()
        for i in range(b):
            idx = torch.nonzero(active[i], as_tuple=True)[0]
            if len(idx) == 0:
                continue
            prev = states[l][i]
            out, _, psi, holo = layers[l](h_curr[i, idx].unsqueeze(0), sssd_state=None if prev is None else prev[0],
                                          cham_hologram=None if prev is None else prev[1])
            h_next[i, idx] = out.squeeze(0)
            states[l][i] = (psi, holo)
        p = acde.compute_halting_probability(h_next)
        if l < min_depth:
            p = torch.zeros_like(p)
        new_acc = acc + p
        halted = (new_acc >= acde.energy_threshold) & active
        still = active & ~halted
        rem = (1.0 - acc).clamp(min=0.0)
        wl = torch.where(halted, rem, p)
        final_h = final_h + (wl * (active | halted).float()).unsqueeze(-1) * h_next
        depth = depth + active.float() + rem * halted.float()
        acc, active, h_curr = new_acc, still, h_next
    if active.any():
        rem = (1.0 - acc).clamp(min=0.0)
        final_h = final_h + (rem * active.float()).unsqueeze(-1) * h_curr
        depth = depth + rem * active.float()
    return final_h, depth, states


def _states_close(a, b):
    for la, lb in zip(a, b):
        for sa, sb in zip(la, lb):
            if sa is None or sb is None:
                assert sa is None and sb is None
                continue
            torch.testing.assert_close(sa[0].reshape(-1), sb[0].reshape(-1), rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(sa[1][0].reshape(-1), sb[1][0].reshape(-1), rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(sa[1][1].reshape(-1), sb[1][1].reshape(-1), rtol=1e-5, atol=1e-6)


def _setup(bias, std, nl=5, seed=0):
    torch.manual_seed(seed)
    layers = nn.ModuleList([RecurrentStandIn(16, seed=10 + l) for l in range(nl)])
    acde = V.AdaptiveCognitiveDepthEngine(hidden_dim=16, energy_threshold=0.99)
    with torch.no_grad():
        acde.w_halting.bias.fill_(bias)
        acde.w_halting.weight.normal_(0.0, std)
    return layers, acde


@pytest.mark.parametrize("bias,std", [(3.0, 0.5), (1.0, 1.5), (-3.0, 0.01)])
def test_batched_loop_equals_the_gathered_loop(bias, std):
    layers, acde = _setup(bias, std)
    x = torch.randn(3, 9, 16)
    with torch.no_grad():
        fh, dc, st = acde.execute_adaptive_recurrent_loop(layers, x, max_depth=12, min_depth=2)
        rfh, rdc, rst = gathered_reference_loop(acde, layers, x, max_depth=12, min_depth=2)
        torch.testing.assert_close(fh, rfh, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(dc, rdc, rtol=0, atol=1e-6)
        _states_close(st, rst)
        # continuation from the returned states with new tokens
        x2 = torch.randn(3, 4, 16)
        fh2, dc2, st2 = acde.execute_adaptive_recurrent_loop(layers, x2, max_depth=12, min_depth=2,
                                                            initial_layer_states=st)
        rfh2, rdc2, rst2 = gathered_reference_loop(acde, layers, x2, max_depth=12, min_depth=2,
                                                   initial_layer_states=rst)
        torch.testing.assert_close(fh2, rfh2, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(dc2, rdc2, rtol=0, atol=1e-6)
        _states_close(st2, rst2)


def test_items_and_layers_that_never_run_keep_their_given_states():
    """Everything halts after min_depth: the later layers' states stay as given (None), and
    an item given states for a layer that halted before it keeps those exact objects."""
    layers, acde = _setup(bias=10.0, std=0.0)
    x = torch.randn(2, 5, 16)
    with torch.no_grad():
        _, _, st = acde.execute_adaptive_recurrent_loop(layers, x, max_depth=12, min_depth=2)
        assert all(st[l][i] is not None for l in range(3) for i in range(2))
        assert all(st[l][i] is None for l in range(3, 5) for i in range(2))
        given = [[None, None] for _ in range(5)]
        marker = (torch.full((1, 1, 2, 2), 7.0), (torch.zeros(1, 2, 2), torch.ones(1, 2, 2)))
        given[4][1] = marker
        _, _, st2 = acde.execute_adaptive_recurrent_loop(layers, x, max_depth=12, min_depth=2,
                                                         initial_layer_states=given)
        assert st2[4][1] is marker and st2[4][0] is None
        _, _, rst2 = gathered_reference_loop(acde, layers, x, max_depth=12, min_depth=2, initial_layer_states=given)
        _states_close(st2, rst2)


def test_max_depth_below_the_layer_count():
    layers, acde = _setup(bias=-3.0, std=0.01)
    x = torch.randn(2, 6, 16)
    with torch.no_grad():
        fh, dc, st = acde.execute_adaptive_recurrent_loop(layers, x, max_depth=3, min_depth=2)
        rfh, rdc, rst = gathered_reference_loop(acde, layers, x, max_depth=3, min_depth=2)
    assert len(st) == 3
    torch.testing.assert_close(fh, rfh, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(dc, rdc, rtol=0, atol=1e-6)
    _states_close(st, rst)
