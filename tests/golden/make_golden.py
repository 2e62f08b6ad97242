"""Generate the golden vectors in this folder by running the REFERENCE implementation.

Run from the repository root in a checkout where the reference package ``verace_v1``
is importable (its source tree on ``PYTHONPATH``, or ``--reference <path>``):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <path-to-Verace-V1>

The reference's eager (pure-PyTorch) path runs on CPU, which is exactly the path its
own tests treat as ground truth (``SSSDAttention.forward`` sssd_attention.py:103-182,
``ContinuousHolographicMemory.forward`` cham_memory.py:117-243,
``newton_schulz_unitary_retraction`` cham_memory.py:21-51).  The cases and seeds follow
the reference's test sweeps (tests/test_triton_kernels.py:86-225, tests/test_cham.py,
tests/test_sssd.py).  Module weights are saved with the inputs so that the oracle and
the CUDA path can be run on exactly the same parameters.

M-CMoE (``ManifoldContinuousMoE.forward`` mcmoe.py:58-120) follows the reference's
tests/test_mcmoe.py shape and the model's configuration (config.py:39-40).

The output files (``sssd_golden.npz``, ``cham_golden.npz``, ``ns_golden.npz``,
``mcmoe_golden.npz``) are committed; the GPU box never runs this script.
"""

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _sd(module):
    return {k: v.detach().cpu().numpy().astype(np.float32) for k, v in module.state_dict().items()}


def _put(store, prefix, **arrays):
    for k, v in arrays.items():
        if v is None:
            continue
        if hasattr(v, "detach"):
            v = v.detach().cpu().numpy()
        store[f"{prefix}/{k}"] = np.asarray(v)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VERACE_REFERENCE", ""))
    ap.add_argument("--only", action="append", choices=["sssd", "cham", "ns", "mcmoe", "layer", "config1", "model"],
                    help="regenerate only these files (default: all)")
    args = ap.parse_args()

    def want(name):
        return not args.only or name in args.only

    if args.reference:
        sys.path.insert(0, args.reference)
    import torch
    from verace_v1.modules.sssd_attention import SSSDAttention
    from verace_v1.modules.cham_memory import (ContinuousHolographicMemory,
                                                newton_schulz_unitary_retraction)
    # one thread: torch 2.11's MKL complex batched solve was seen to spin forever with an
    # explicit multi-thread setting on this host (CLASWP parameter errors).
    if args.only not in (["config1"], ["model"]):
        torch.set_num_threads(1)

    if want("sssd"):
        # ------------------------------------------------------------------ SSSD
        sssd = {}
        cases = []
        # shape sweep of tests/test_triton_kernels.py:86-106 (seed 0)
        for (b, s, d, h) in [(2, 8, 16, 2), (1, 1, 16, 1), (2, 13, 16, 2), (2, 8, 24, 2)]:
            cases.append((f"sweep_b{b}_s{s}_d{d}_h{h}", 0, b, s, d, h, h * d, None))
        # halted back half (tests/test_triton_kernels.py:109-125, seed 1)
        cases.append(("halted", 1, 2, 10, 16, 2, 32, "back_half"))
        # production head size, small hidden width (weights stay small)
        cases.append(("d128", 11, 1, 16, 128, 2, 16, None))
        cases.append(("d64_norm", 12, 2, 8, 64, 2, 128, None))  # tests/test_sssd.py:10-26 shape
        for name, seed, b, s, d, h, hid, mask_kind in cases:
            torch.manual_seed(seed)
            m = SSSDAttention(hidden_dim=hid, num_heads=h, head_dim=d)
            x = torch.randn(b, s, hid)
            mask = None
            if mask_kind == "back_half":
                mask = torch.ones(b, s, dtype=torch.bool)
                mask[:, s // 2:] = False
            with torch.no_grad():
                out, state = m(x, return_state=True, active_mask=mask)
            _put(sssd, name, x=x, out=out, state=state, mask=mask,
                 dims=np.array([b, s, d, h, hid]))
            for k, v in _sd(m).items():
                sssd[f"{name}/p/{k}"] = v
        # initial_state round trip (tests/test_triton_kernels.py:128-148, seed 2)
        torch.manual_seed(2)
        b, s, d, h = 2, 6, 16, 2
        m = SSSDAttention(hidden_dim=h * d, num_heads=h, head_dim=d)
        x1 = torch.randn(b, s, h * d)
        x2 = torch.randn(b, s, h * d)
        with torch.no_grad():
            out1, st1 = m(x1, return_state=True)
            out2, st2 = m(x2, initial_state=st1, return_state=True)
        _put(sssd, "roundtrip", x1=x1, x2=x2, out1=out1, state1=st1, out2=out2, state2=st2,
             dims=np.array([b, s, d, h, h * d]))
        for k, v in _sd(m).items():
            sssd[f"roundtrip/p/{k}"] = v
        np.savez_compressed(os.path.join(HERE, "sssd_golden.npz"), **sssd)

    if want("cham"):
        # ------------------------------------------------------------------ CHAM
        cham = {}
        cases = []
        # shape sweep of tests/test_triton_kernels.py:151-173 (seed 3, hidden 32)
        for (b, s, D) in [(2, 8, 16), (1, 1, 16), (2, 5, 16), (2, 8, 20), (2, 6, 160)]:
            cases.append((f"sweep_b{b}_s{s}_D{D}", 3, b, s, D, 32, None))
        cases.append(("halted", 4, 2, 10, 16, 32, "back_half"))      # :176-197
        cases.append(("zero_gamma", 5, 2, 12, 16, 32, "all_off"))    # :200-223
        cases.append(("long_s100", 7, 2, 100, 16, 32, None))         # :243-275
        cases.append(("D64_s64", 13, 2, 64, 64, 64, None))
        for name, seed, b, s, D, hid, mask_kind in cases:
            print("cham case", name, flush=True)
            torch.manual_seed(seed)
            m = ContinuousHolographicMemory(hidden_dim=hid, holographic_dim=D)
            x = torch.randn(b, s, hid)
            mask = None
            if mask_kind == "back_half":
                mask = torch.ones(b, s, dtype=torch.bool)
                mask[:, s // 2:] = False
            elif mask_kind == "all_off":
                mask = torch.zeros(b, s, dtype=torch.bool)
            with torch.no_grad():
                y, (Hr, Hi) = m(x, active_mask=mask)
            _put(cham, name, x=x, out=y, Hr=Hr, Hi=Hi, mask=mask, dims=np.array([b, s, D, hid]))
            for k, v in _sd(m).items():
                cham[f"{name}/p/{k}"] = v
        # initial_hologram round trip: two chunks through initial_hologram
        torch.manual_seed(8)
        b, s, D, hid = 2, 7, 24, 32
        m = ContinuousHolographicMemory(hidden_dim=hid, holographic_dim=D)
        x1 = torch.randn(b, s, hid)
        x2 = torch.randn(b, s, hid)
        with torch.no_grad():
            y1, H1 = m(x1)
            y2, H2 = m(x2, initial_hologram=H1)
        _put(cham, "roundtrip", x1=x1, x2=x2, out1=y1, Hr1=H1[0], Hi1=H1[1], out2=y2,
             Hr2=H2[0], Hi2=H2[1], dims=np.array([b, s, D, hid]))
        for k, v in _sd(m).items():
            cham[f"roundtrip/p/{k}"] = v
        # non-unitary initial hologram (exercises the readout retraction of H_0)
        torch.manual_seed(9)
        b, s, D, hid = 2, 5, 16, 32
        m = ContinuousHolographicMemory(hidden_dim=hid, holographic_dim=D)
        x = torch.randn(b, s, hid)
        H0r = torch.eye(D).expand(b, D, D) + 0.05 * torch.randn(b, D, D)
        H0i = 0.05 * torch.randn(b, D, D)
        with torch.no_grad():
            y, (Hr, Hi) = m(x, initial_hologram=(H0r, H0i))
        _put(cham, "nonunitary_h0", x=x, H0r=H0r, H0i=H0i, out=y, Hr=Hr, Hi=Hi,
             dims=np.array([b, s, D, hid]))
        for k, v in _sd(m).items():
            cham[f"nonunitary_h0/p/{k}"] = v
        # production holographic width D = 1024 (small hidden so the weights stay small);
        # the 8 MiB state is summarised by its first rows, diagonal and column sums.
        torch.manual_seed(10)
        b, s, D, hid = 1, 3, 1024, 16
        m = ContinuousHolographicMemory(hidden_dim=hid, holographic_dim=D)
        x = torch.randn(b, s, hid)
        with torch.no_grad():
            y, (Hr, Hi) = m(x)
        _put(cham, "D1024", x=x, out=y, dims=np.array([b, s, D, hid]),
             Hr_rows=Hr[:, :4], Hi_rows=Hi[:, :4],
             Hr_diag=torch.diagonal(Hr, dim1=-2, dim2=-1), Hi_diag=torch.diagonal(Hi, dim1=-2, dim2=-1),
             Hr_colsum=Hr.sum(-2), Hi_colsum=Hi.sum(-2))
        for k, v in _sd(m).items():
            cham[f"D1024/p/{k}"] = v
        np.savez_compressed(os.path.join(HERE, "cham_golden.npz"), **cham)

    if want("ns"):
        # ------------------------------------------------------------------ NS retraction
        ns = {}
        torch.manual_seed(0)  # tests/test_cham.py:129-160
        d = 16
        Hr = torch.randn(2, d, d) * 0.1 + torch.eye(d)
        Hi = torch.randn(2, d, d) * 0.1
        r, i = newton_schulz_unitary_retraction(Hr.clone(), Hi.clone())
        _put(ns, "d16", Hr=Hr, Hi=Hi, out_r=r, out_i=i)
        torch.manual_seed(1)
        d = 160
        Hr = torch.randn(1, d, d) * 0.02 + torch.eye(d)
        Hi = torch.randn(1, d, d) * 0.02
        r, i = newton_schulz_unitary_retraction(Hr.clone(), Hi.clone())
        _put(ns, "d160", Hr=Hr, Hi=Hi, out_r=r, out_i=i)
        np.savez_compressed(os.path.join(HERE, "ns_golden.npz"), **ns)
    if want("mcmoe"):
        # ------------------------------------------------------------------ M-CMoE
        from verace_v1.modules.mcmoe import ManifoldContinuousMoE
        mc = {}
        # the reference test's shape (tests/test_mcmoe.py:8-12) and the model's M-CMoE
        # (config.py: rank 32, 64 components, top-8) at hidden 256 and 1024
        for name, b, s, d, rank, C, K in [("t256", 2, 8, 256, 16, 8, 8), ("m256", 2, 12, 256, 32, 64, 8),
                                          ("m1024", 1, 16, 1024, 32, 64, 8)]:
            torch.manual_seed(0)
            m = ManifoldContinuousMoE(hidden_dim=d, rank=rank, num_components=C, top_k_components=K)
            torch.manual_seed(1)
            x = torch.randn(b, s, d)
            with torch.no_grad():
                y = m(x)
                xf = x.reshape(b * s, d)
                base = m.base_w_down(m.base_situ_glu(xf))
                logits = m.router(xf)
                # the routing lines of mcmoe.py:91-96, for the intermediate values
                tl, ti = torch.topk(logits, k=min(K, C), dim=-1)
                masked = torch.full_like(logits, float("-inf"))
                masked.scatter_(-1, ti, tl)
                tw = torch.gather(torch.softmax(masked, dim=-1), -1, ti)
            _put(mc, name, x=x, y=y, base=base, logits=logits, topk_idx=ti, topk_w=tw,
                 dims=np.array([b, s, d, rank, C, K]))
            # the weights themselves are re-created by the tests (same constructor, seed 0);
            # a fingerprint of each (sum, sum of squares, first 16 values) pins them
            for k, v in _sd(m).items():
                f = v.astype(np.float64).ravel()
                mc[f"{name}/fp/{k}"] = np.concatenate([[f.sum(), (f * f).sum()], f[:16]])
        np.savez_compressed(os.path.join(HERE, "mcmoe_golden.npz"), **mc)
    if want("layer"):
        # ------------------------------------------------------------------ layer + ACDE
        # VeraceV1Layer.forward (backbone.py:53-101) and
        # AdaptiveCognitiveDepthEngine.execute_adaptive_recurrent_loop (acd_engine.py:36-167)
        # at a small configuration (head_dim 128 and D = 256, the widths the tensor-core
        # paths take).  States are stored as sketches: psi @ r (r a fixed random vector)
        # and H @ r, which the tests form from their own states.
        from verace_v1.config import VeraceV1Config
        from verace_v1.modules.backbone import VeraceV1Layer
        from verace_v1.modules.acd_engine import AdaptiveCognitiveDepthEngine
        ly = {}
        cfg = VeraceV1Config(vocab_size=100, hidden_dim=256, num_layers=4, num_heads=2, head_dim=128,
                             spectral_dim=64, chams_holographic_dim=256, mcmoe_rank=16, mcmoe_num_components=8)
        g = torch.Generator().manual_seed(5)
        r_d = torch.randn(128, generator=g)
        r_D = torch.randn(256, generator=g)
        ly["sketch/r_d"] = r_d.numpy()
        ly["sketch/r_D"] = r_D.numpy()

        def sk(prefix, psi, holo):
            _put(ly, prefix, psi_r=psi @ r_d, hr_r=holo[0] @ r_D, hi_r=holo[1] @ r_D)

        torch.manual_seed(0)
        layers = torch.nn.ModuleList([VeraceV1Layer(i, cfg) for i in range(4)])
        acde = AdaptiveCognitiveDepthEngine(hidden_dim=256, energy_threshold=0.99)
        with torch.no_grad():   # halting that varies per token: some halt at layer 2, most at 3
            acde.w_halting.bias.fill_(3.0)
            acde.w_halting.weight.normal_(0.0, 0.2, generator=g)
        ly["acde/w_halting.weight"] = acde.w_halting.weight.detach().numpy()
        ly["acde/w_halting.bias"] = acde.w_halting.bias.detach().numpy()
        torch.manual_seed(1)
        x = torch.randn(2, 16, 256)
        mask = torch.ones(2, 16, dtype=torch.bool)
        mask[0, 3] = mask[1, 10:] = False
        with torch.no_grad():
            # layer 0: snapshot commit, fresh states
            h1, br1, s1, c1 = layers[0](x)
            _put(ly, "L0", x=x, h=h1, br=br1)
            sk("L0", s1, c1)
            # layer 1: AttnRes mixing over br1, carried states, partial active mask
            h2, br2, s2, c2 = layers[1](h1, block_residual=br1, sssd_state=s1, cham_hologram=c1, active_mask=mask)
            _put(ly, "L1", h=h2, br=br2, mask=mask)
            sk("L1", s2, c2)
            # ACDE over the four layers, then a continuation with 4 new tokens
            torch.manual_seed(2)
            xa = torch.randn(2, 12, 256)
            fh, dc, st = acde.execute_adaptive_recurrent_loop(layers, xa, max_depth=12, min_depth=2)
            _put(ly, "A0", x=xa, final_h=fh, depth=dc)
            for l in range(4):
                for i in range(2):
                    if st[l][i] is None:
                        ly[f"A0/none_{l}_{i}"] = np.array(1)
                    else:
                        sk(f"A0/s{l}_{i}", st[l][i][0], st[l][i][1])
            xb = torch.randn(2, 4, 256)
            fh2, dc2, st2 = acde.execute_adaptive_recurrent_loop(layers, xb, max_depth=12, min_depth=2,
                                                                 initial_layer_states=st)
            _put(ly, "A1", x=xb, final_h=fh2, depth=dc2)
            for l in range(4):
                for i in range(2):
                    if st2[l][i] is not None:
                        sk(f"A1/s{l}_{i}", st2[l][i][0], st2[l][i][1])
        for k, v in _sd(layers).items():
            f = v.astype(np.float64).ravel()
            ly[f"layers/fp/{k}"] = np.concatenate([[f.sum(), (f * f).sum()], f[:16]])
        np.savez_compressed(os.path.join(HERE, "layer_golden.npz"), **ly)
    if want("config1"):
        # ------------------------------------------------------------------ config 1, full size
        # One SSSD + CHAM layer in fp32 at the benchmark configuration: hidden 1024, 8 heads x
        # 128, D = 1024, x = randn(2, 512, 1024) under seed 0, weights default-initialised
        # under seed 0 (SSSDAttention first, then ContinuousHolographicMemory, both fed x).
        # The reference's eager CHAM needs ~16 GB per 64 tokens at D = 1024, so it runs in
        # 64-token chunks through initial_hologram (the state composes exactly on the right,
        # cham_memory.py:222-230).  Outputs and states are stored as sketches (products with
        # fixed random matrices stored here) plus full rows at a few positions; weights and
        # x as fingerprints (the tests rebuild them from the same seeds).
        import time
        c1 = {}   # run alone (--only config1): torch's default thread count
        torch.manual_seed(0)
        sssd_m = SSSDAttention(1024, 8, 128, 256)
        cham_m = ContinuousHolographicMemory(1024, 1024)
        torch.manual_seed(0)
        x = torch.randn(2, 512, 1024)
        g = torch.Generator().manual_seed(21)
        r_out = torch.randn(1024, 8, generator=g)
        r_d = torch.randn(128, 4, generator=g)
        r_D = torch.randn(1024, 4, generator=g)
        rows = torch.tensor([0, 1, 63, 64, 127, 200, 255, 256, 383, 511])
        c1["sketch/r_out"] = r_out.numpy()
        c1["sketch/r_d"] = r_d.numpy()
        c1["sketch/r_D"] = r_D.numpy()
        c1["sketch/rows"] = rows.numpy()

        def fp(t):
            f = t.detach().double().reshape(-1)
            return torch.cat([torch.stack([f.sum(), (f * f).sum()]), f[:16]]).numpy()

        c1["x/fp"] = fp(x)
        for k, v in sssd_m.state_dict().items():
            c1[f"sssd/fp/{k}"] = fp(v)
        for k, v in cham_m.state_dict().items():
            c1[f"cham/fp/{k}"] = fp(v)
        with torch.no_grad():
            t0 = time.time()
            out, psi = sssd_m(x, return_state=True)
            print("config1 sssd", time.time() - t0, "s", flush=True)
            _put(c1, "sssd", out_sk=out @ r_out, out_rows=out[:, rows], psi_sk=psi @ r_d,
                 psi_diag=torch.diagonal(psi, dim1=-2, dim2=-1))
            H = None
            ys = []
            for c0 in range(0, 512, 64):
                t0 = time.time()
                y, H = cham_m(x[:, c0:c0 + 64], initial_hologram=H)
                ys.append(y)
                print("config1 cham chunk", c0, time.time() - t0, "s", flush=True)
            y = torch.cat(ys, dim=1)
            Hr, Hi = H
            _put(c1, "cham", out_sk=y @ r_out, out_rows=y[:, rows], hr_sk=Hr @ r_D, hi_sk=Hi @ r_D,
                 hr_diag=torch.diagonal(Hr, dim1=-2, dim2=-1), hi_diag=torch.diagonal(Hi, dim1=-2, dim2=-1))
        np.savez_compressed(os.path.join(HERE, "config1_golden.npz"), **c1)
    if want("model"):
        # ------------------------------------------------------------------ the model
        # VeraceV1Model.forward (backbone.py:144-210) at a small configuration (head_dim 128,
        # D = 128: the tensor-core widths): ACDE prefill of 2 x 12 tokens, then two
        # single-token steps through layer_states (the decode convention of
        # serving/hyper_generate.py:58-77).  The in-path weights are re-initialised by
        # tests/conftest.py:model_reinit (the tests re-create them the same way) and pinned
        # by fingerprints; the vision encoder is built small and never used.
        sys.path.insert(0, os.path.dirname(HERE))
        from conftest import model_fingerprints, model_reinit
        from verace_v1.config import VeraceV1Config
        from verace_v1.modules.backbone import VeraceV1Model

        @__import__("dataclasses").dataclass
        class TinyVision:
            embed_dim: int = 32
            num_layers: int = 1
            num_heads: int = 2
            patch_size: int = 14

        cfg = VeraceV1Config(vocab_size=64, hidden_dim=128, num_layers=4, num_heads=1, head_dim=128,
                             spectral_dim=64, chams_holographic_dim=128, mcmoe_rank=8, mcmoe_num_components=8,
                             vision_config=TinyVision())
        torch.manual_seed(0)
        model = VeraceV1Model(cfg).eval()
        model_reinit(model, seed=0)
        md = {}
        for k, v in model_fingerprints(model).items():
            md[f"fp/{k}"] = v
        ids = torch.randint(0, 64, (2, 12), generator=torch.Generator().manual_seed(1))
        nxt = torch.randint(0, 64, (2, 2), generator=torch.Generator().manual_seed(2))
        with torch.no_grad():
            logits, depth, hidden, st = model(ids, return_hidden=True, return_layer_states=True)
            md["prefill/ids"] = ids.numpy()
            md["prefill/logits"] = logits.numpy()
            md["prefill/depth"] = depth.numpy()
            md["prefill/hidden"] = hidden.numpy()
            for i in range(2):
                lg, dp, st = model(nxt[:, i:i + 1], layer_states=st, return_layer_states=True)
                md[f"step{i}/ids"] = nxt[:, i:i + 1].numpy()
                md[f"step{i}/logits"] = lg.numpy()
                md[f"step{i}/depth"] = dp.numpy()
            lg, dp = model(ids, use_adaptive_depth=False)
            md["static/logits"] = lg.numpy()
        np.savez_compressed(os.path.join(HERE, "model_golden.npz"), **md)
    for f in ("sssd_golden.npz", "cham_golden.npz", "ns_golden.npz", "mcmoe_golden.npz", "layer_golden.npz",
              "config1_golden.npz", "model_golden.npz"):
        if os.path.exists(os.path.join(HERE, f)):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
