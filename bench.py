#!/usr/bin/env python
"""Benchmark of the Verace V1 SSSD + CHAM sequence-mixing path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark config 2): the SSSD and CHAM sublayers of a 12-layer Verace V1
stack (hidden 1024, 8 heads x 128, holographic width 1024) over a prefill batch of
8 sequences x 2048 tokens in bf16 (fp32 recurrent state), random-init weights
(seed 0), synthetic token embeddings (uniform ids over [0, 32000), seed 0).  One
step = every layer's h <- h + SSSD(RMSNorm(h)); h <- h + CHAM(RMSNorm(h)), through
the package's module API (projections on cuBLAS, scans, RMSNorms and residual adds on the
sm_100a kernels).
The M-CMoE FFN and ACDE halting are outside this path; random-init ACDE halts no
token before layer 12, so every token runs all 12 layers.

Unit: token-layers/s (one token through SSSD + CHAM of one layer).

Decode (benchmark config 3, reported under "decode"): the same 12 layers, 64 items per
GPU, a 1024-token prompt prefilled with the scans, then 256 single-token steps with
teacher-forced random ids, each step one CUDA graph of the layer glue and the decode
kernels that update the resident states in place (verace_decode_step for the SSSD heads;
verace_decode_cham_lazy for the holograms: one read of each hologram per step, the rank-2
updates deferred and folded in every 8th step).  Reported as µs per step and µs per token
(= step / 64).

Multi-GPU (torchrun, one rank per GPU): each rank runs the full config-2 batch on its
own items (weak scaling: batch shards, no collective on the data path); time is the
max over ranks of the CUDA-event time.

--impl reference times the reference's CPU algorithm (the eager path, restated in
numpy by oracle/) on this host's cores, on a bounded sample of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SSSD+CHAM scan tokens/s at 1/2/4/8 B200 + % roofline; decode step µs/token"
UNIT = "token-layers/s"
CFG = dict(layers=12, batch=8, seq=2048, hidden=1024, heads=8, head_dim=128, holo=1024, vocab=32000)
DEC = dict(batch=64, prompt=1024, steps=256, pending=8)


def build_chain(V, dev):
    """The config-2/3 chain: per layer RMSNorm -> SSSD -> RMSNorm -> CHAM (bf16 weights,
    random init from seed 0), and the token embedding."""
    import torch
    c = CFG
    dt = torch.bfloat16
    torch.manual_seed(0)
    layers = []
    for _ in range(c["layers"]):
        layers.append(torch.nn.ModuleDict(dict(
            sssd_norm=torch.nn.RMSNorm(c["hidden"], eps=1e-6),
            sssd=V.SSSDAttention(c["hidden"], c["heads"], c["head_dim"], 256),
            cham_norm=torch.nn.RMSNorm(c["hidden"], eps=1e-6),
            cham=V.ContinuousHolographicMemory(c["hidden"], c["holo"]))).to(dev, dt).eval())
    embed = torch.nn.Embedding(c["vocab"], c["hidden"]).to(dev, dt)
    return layers, embed


def _load_package():
    import importlib.util
    if "verace_v1_b200" in sys.modules:
        return sys.modules["verace_v1_b200"]
    pkg = os.path.join(ROOT, "verace-v1_b200")
    spec = importlib.util.spec_from_file_location("verace_v1_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["verace_v1_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------------------ ranks
def rank_shard_ids(rank, batch, seq, vocab):
    """The rank's shard of the synthetic prefill batch: `batch` sequences of `seq` token
    ids from a generator seeded by the rank (weak scaling: every rank has the same amount
    of work on items of its own; no data crosses ranks)."""
    import torch
    gen = torch.Generator().manual_seed(0 + rank)
    return torch.randint(0, vocab, (batch, seq), generator=gen)


def make_rank_sync(world, device):
    """(barrier, max_over_ranks) for the current process group.  On a CUDA device both
    synchronise the device around the collective, so the timed region is bracketed on
    every rank; max_over_ranks reduces one float (a time in ms) to its maximum."""
    import torch
    import torch.distributed as dist
    cuda = device.type == "cuda"

    def barrier():
        if cuda:
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if cuda:
            torch.cuda.synchronize()

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    return barrier, max_over_ranks


def whole_job_rate(world, units_per_rank_step, ms_per_step):
    """Units all ranks processed per second, over the slowest rank's time per step."""
    return world * units_per_rank_step / (ms_per_step * 1e-3)


def gather_outputs(world, t):
    """Every rank's output shard, concatenated along dim 0 on every rank (one NCCL
    all_gather over NVLink; the only data-path collective: the items are independent)."""
    if world == 1:
        return t
    import torch
    import torch.distributed as dist
    out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous())
    return out


def strong_shard(rank, world, global_batch):
    """The contiguous range [lo, hi) of a fixed global batch's items that a rank runs
    (strong scaling: the total work is fixed, each rank takes a share)."""
    per = (global_batch + world - 1) // world
    lo = min(rank * per, global_batch)
    return lo, min(lo + per, global_batch)


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={','.join(self.FIELDS)}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist
    V = _load_package()
    from verace_v1_b200 import _lib
    from verace_v1_b200.kernels import launch_cham_update, launch_sssd_scan

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    c = CFG
    layers, embed = build_chain(V, dev)
    ids = rank_shard_ids(rank, c["batch"], c["seq"], c["vocab"]).to(dev)
    with torch.no_grad():
        x = embed(ids).contiguous()

    cham_events = []

    def step(h, record=False, inplace=False):
        # the residual stream h is updated in place by the fused residual + RMSNorm glue:
        # h <- h + SSSD(n), n <- RMSNorm(h); h <- h + RMSNorm(CHAM(n)), n <- next pre-norm
        if not inplace:
            h = h.clone()
        n = V.rmsnorm(h, layers[0]["sssd_norm"])
        for li, L in enumerate(layers):
            o, _ = L["sssd"](n, return_state=True)
            n = V.add_rmsnorm(h, o, out_norm=L["cham_norm"])
            cm = L["cham"]
            q, k, v, g = cm.project(n)
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
            rec, _ = launch_cham_update(q, k, v, g)
            if record:
                e1.record()
                cham_events.append((e0, e1))
            nxt = layers[li + 1]["sssd_norm"] if li + 1 < len(layers) else None
            n = V.add_rmsnorm(h, cm.w_out(rec), y_norm=cm.norm, out_norm=nxt)
        gather_outputs(world, h)     # every rank receives all ranks' outputs (NCCL all_gather)
        return h

    barrier, max_over_ranks = make_rank_sync(world, dev)

    tokens_per_step = c["batch"] * c["seq"] * c["layers"]
    with torch.no_grad():
        for _ in range(args.warmup):
            step(x)
        barrier()
        gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
        sampler = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}")
        sampler.start()
        time.sleep(0.3)
        launches0 = _lib.lib().verace_kernel_launches()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record()
        for _ in range(args.steps):
            step(x, record=True)
        e_end.record()
        barrier()
        launches = _lib.lib().verace_kernel_launches() - launches0
        clocks = sampler.stop()
        ms = max_over_ranks(e_start.elapsed_time(e_end)) / args.steps
        cham_ms = statistics.mean(a.elapsed_time(b) for a, b in cham_events)

        # end to end through the public API: every step's input copied from pinned host memory
        # and its result read back, double-buffered as a serving loop does: a copy stream brings
        # step i+1's input in and takes step i's result out while step i / i+1 compute (all
        # copies inside the timed region)
        x_host = x.cpu().pin_memory()
        out_host = torch.empty_like(x_host).pin_memory()
        main = torch.cuda.current_stream(dev)
        copy = torch.cuda.Stream(dev)
        xin = [torch.empty_like(x) for _ in range(2)]

        def e2e_steps(n):
            ev_in = [torch.cuda.Event() for _ in range(2)]
            ev_done = [torch.cuda.Event() for _ in range(2)]
            copy.wait_stream(main)
            with torch.cuda.stream(copy):
                xin[0].copy_(x_host, non_blocking=True)
                ev_in[0].record(copy)
            for i in range(n):
                bcur = i % 2
                main.wait_event(ev_in[bcur])
                step(xin[bcur], inplace=True)           # the residual stream, updated in place
                ev_done[bcur].record(main)
                with torch.cuda.stream(copy):
                    if i + 1 < n:                        # (after the previous read-out of that buffer)
                        xin[(i + 1) % 2].copy_(x_host, non_blocking=True)
                        ev_in[(i + 1) % 2].record(copy)
                    copy.wait_event(ev_done[bcur])
                    out_host.copy_(xin[bcur], non_blocking=True)
            main.wait_stream(copy)

        e2e_steps(max(1, args.warmup // 2))
        barrier()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record()
        e2e_steps(args.steps)
        e3.record()
        barrier()
        e2e_ms = max_over_ranks(e2.elapsed_time(e3)) / args.steps

    hbm, bf16_burst, bf16_sus, peak_kind = _peaks()
    D, b, s = c["holo"], c["batch"], c["seq"]
    nch = (s + 63) // 64
    # Roofline of one verace_cham_scan call on the algorithmic basis of the path's work
    # unit: FLOP = the necessary 18 D^2 per token (9 D^2 MAC: the rank-2 state update 8 D^2
    # and the readout D^2; the reference formulation's 228 D^2 includes a per-position
    # Newton-Schulz polynomial that is the identity for the fresh hologram and is not
    # counted), bytes = the state read and written once per call (2 planes x D^2 x 4 B,
    # each way) plus q, k, v in and the readout out in bf16 and gamma in fp32 per token.
    # T_roof = max(bytes / HBM peak, FLOP / sustained bf16 peak); the call is tensor-bound.
    cham_flop = 18.0 * D * D * b * s
    cham_bytes_algo = b * 2 * (2 * D * D * 4) + b * s * (4 * D * 2 + 4)
    t_meas = cham_ms * 1e-3
    t_roof = max(cham_bytes_algo / (hbm * 1e9), cham_flop / (bf16_sus * 1e12))
    tflops = cham_flop / t_meas / 1e12
    # This design's own traffic: the chunked scan reads and writes the D x D complex state
    # once per 64-token chunk (the identity start is not read), and moves q/k/v/readout and
    # the per-chunk T coefficients (128 KB per item and chunk, written by the prep, read by
    # the column pass).  DRAM bytes per (item, chunk) measured by ncu at b=16, s=256
    # (profiles/cham_tc_colpass2_b16_s256.md 887.6 MB per column-pass launch;
    # cham_tc_readout_batch_b16_s256.md 304.1 MB per readout launch; cham_tc_prep_ws_b16_s256.md
    # 16.8 MB per prep launch, 64 item-chunks each), scaled to this call.
    chunk_bytes = (2 * nch - 1) * b * 2 * D * D * 4 + 4 * b * s * D * 2 + 2 * nch * b * 131072
    traffic = (887.6e6 + 304.1e6 + 16.8e6) / 64 * b * nch
    result = {
        "metric": METRIC, "value": whole_job_rate(world, tokens_per_step, ms), "unit": UNIT,
        "model_tokens_per_s": whole_job_rate(world, c["batch"] * c["seq"], ms),   # through all 12 layers
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (fp32 recurrent state)", "data": "synthetic",
        "config": {"workload": "config 2: 12-layer SSSD+CHAM prefill, b=8 x s=2048 per GPU, "
                               "hidden 1024, 8x128 heads, D=1024",
                   "global_batch": b * world, "seq_len": s, "layers": c["layers"],
                   "parallelism": f"dp{world} (batch shards; outputs all-gathered over NCCL each step)",
                   "l2": "no flush: per-step working set (weights 190 MB + activations) > 126 MB L2"},
        "roofline": {"kernel": "verace_cham_scan (cham_tc_prep_ws, then per group of 12 chunks one cham_tc_colpass2 "
                               "and one cham_tc_readout_batch)",
                     "bound": "tensor", "achieved": tflops, "peak": bf16_sus, "unit": "TFLOP/s",
                     "frac": t_roof / t_meas, "traffic": traffic,
                     "basis": "18 D^2 FLOP per token-layer (necessary: rank-2 update + readout); bytes = state "
                              "read+written once per call + (4 D + 1) elements per token; "
                              "frac = max(bytes/HBM, FLOP/bf16 sustained) / measured",
                     "flop_per_launch": cham_flop, "bytes_per_launch": cham_bytes_algo,
                     "t_roof_ms": t_roof * 1e3, "ms_per_launch": cham_ms,
                     "peak_source": f"{peak_kind} cuBLAS bf16 GEMM, sustained (MEASURED_PEAKS.json); "
                                    f"HBM {hbm} GB/s {peak_kind} copy",
                     "frac_of_bf16_burst": tflops / bf16_burst,
                     "reference_formulation_flop": 228.0 * D * D * b * s,
                     "chunked_design": {"bytes_per_launch": chunk_bytes, "unit": "GB/s",
                                        "achieved": chunk_bytes / t_meas / 1e9, "peak": hbm,
                                        "frac": chunk_bytes / t_meas / 1e9 / hbm,
                                        "note": "this design's own bytes: the state read and written once per "
                                                "64-token chunk"}},
        "e2e": {"value": whole_job_rate(world, tokens_per_step, e2e_ms), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * x.element_size(),
                "d2h_bytes_per_step": x.numel() * x.element_size()},
        "clocks": clocks,
        "gpu_launches": int(launches),
    }
    if not args.no_decode:
        del x
        torch.cuda.empty_cache()
        result["decode"] = run_decode(args, layers, embed, V, dev, rank, barrier, max_over_ranks)
    if not args.no_mcmoe:
        torch.cuda.empty_cache()
        result["mcmoe"] = run_mcmoe(args, V, dev, barrier, max_over_ranks)
    if not args.no_model:
        torch.cuda.empty_cache()
        result["model"] = run_model(args, V, dev, rank, world, barrier, max_over_ranks)
    if not args.no_strong:
        torch.cuda.empty_cache()
        result["strong"] = run_strong(args, V, dev, rank, world, barrier, max_over_ranks)
    if not args.no_long:
        torch.cuda.empty_cache()
        result["long"] = run_long(args, V, dev, rank, world, barrier, max_over_ranks)
    if world == 1 and not args.no_decode and not args.no_triton_bar:
        torch.cuda.empty_cache()
        result["decode"]["reference_triton"] = run_triton_bar(dev)
        torch.cuda.empty_cache()
        result["c1_scans"] = run_triton_c1(V, dev)
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_sample(tokens=args.cpu_tokens)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_model(args, V, dev, rank, world, barrier, max_over_ranks):
    """benchmark config 2 as the whole model: VeraceV1Model (12 layers of SSSD + CHAM +
    M-CMoE, ACDE halting at the default configuration, the LM head) prefill of the rank's
    8 x 2048 uniform-random ids, random init (seed 0), weights in bf16, through the drop-in
    model's forward.  Tokens/s over all ranks; the headline line times the SSSD + CHAM
    chain of the same layers alone."""
    import torch
    c = CFG
    cfg = V.VeraceV1Config(vocab_size=c["vocab"], hidden_dim=c["hidden"], num_layers=c["layers"],
                           num_heads=c["heads"], head_dim=c["head_dim"], chams_holographic_dim=c["holo"])
    torch.manual_seed(0)
    model = V.VeraceV1Model(cfg).to(dev, torch.bfloat16).eval()
    ids = rank_shard_ids(rank, c["batch"], c["seq"], c["vocab"]).to(dev)
    with torch.no_grad():
        for _ in range(max(1, min(args.warmup, 2))):
            logits, depth = model(ids)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 2
        e0.record()
        for _ in range(reps):
            logits, depth = model(ids)
        e1.record()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / reps)
        mean_depth = float(depth.float().mean())
    del model, logits
    tokens = world * c["batch"] * c["seq"]
    return {"workload": "config 2 as VeraceV1Model: 12 layers (SSSD + CHAM + M-CMoE top-8/64), ACDE at the "
                        "default config, LM head; b=8 x s=2048 per GPU, bf16 weights, random init",
            "ms_per_forward": ms, "model_tokens_per_s": tokens / (ms * 1e-3),
            "mean_ponder_cost": mean_depth}


C5 = dict(batch=256, seq=4096, hidden=4096, heads=32, head_dim=128, holo=1024, vocab=32000, micro=8)


def run_strong(args, V, dev, rank, world, barrier, max_over_ranks):
    """Config 5, one decoder layer, strong scaling: a fixed global batch of 256 sequences x
    4096 uniform-random token ids (seed 0) through one VeraceV1Layer (SSSD 32 heads x 128,
    CHAM D = 1024, M-CMoE rank 32 / 64 components / top-8; hidden 4096; random init, seed 0;
    bf16 activations, fp32 recurrent states), the items split across the ranks (256/N each),
    run in micro-batches of 8 items.  Each step ends with the NCCL all_gather of every
    item's last-position hidden state (the outputs a generation step reads).  Time: the
    max over ranks of the CUDA-event time per step.  The 32-layer model is 32 x this work
    per forward (ACDE halting at random init keeps every token for all layers)."""
    import torch
    c = C5
    cfg = V.VeraceV1Config(vocab_size=c["vocab"], hidden_dim=c["hidden"], num_layers=1, num_heads=c["heads"],
                           head_dim=c["head_dim"], chams_holographic_dim=c["holo"])
    torch.manual_seed(0)
    layer = V.VeraceV1Layer(1, cfg).to(dev, torch.bfloat16).eval()   # layer_idx 1: no snapshot commit
    embed = torch.nn.Embedding(c["vocab"], c["hidden"]).to(dev, torch.bfloat16)
    ids = torch.randint(0, c["vocab"], (c["batch"], c["seq"]), generator=torch.Generator().manual_seed(0))
    lo, hi = strong_shard(rank, world, c["batch"])
    ids = ids[lo:hi].to(dev)
    last = torch.empty(hi - lo, c["hidden"], device=dev, dtype=torch.bfloat16)

    def step():
        for m0 in range(0, hi - lo, c["micro"]):
            x = embed(ids[m0:m0 + c["micro"]])
            h, _, _, _ = layer(x)
            last[m0:m0 + c["micro"]].copy_(h[:, -1])
        return gather_outputs(world, last)

    with torch.no_grad():
        for _ in range(max(1, min(args.warmup, 2))):
            step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 2
        e0.record()
        for _ in range(reps):
            out = step()
        e1.record()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / reps)
    assert out.shape[0] == c["batch"]
    del layer, embed
    tokens = c["batch"] * c["seq"]
    return {"workload": "config 5, one VeraceV1Layer (SSSD 32x128 + CHAM D=1024 + M-CMoE top-8/64), hidden 4096, "
                        "global batch 256 x 4096 tokens split over the ranks (strong scaling), bf16, micro-batches "
                        "of 8 items, last-position hidden states all-gathered each step",
            "scaling": "strong", "n_gpus": world, "items_per_rank": hi - lo, "ms_per_step": ms,
            "token_layers_per_s": tokens / (ms * 1e-3),
            "model_tokens_per_s_32_layers": tokens / (32 * ms * 1e-3)}


C4 = dict(seq=65536, hidden=2048, heads=16, head_dim=128, holo=1024)


def run_long(args, V, dev, rank, world, barrier, max_over_ranks):
    """Config 4: one long sequence through one layer's SSSD and CHAM sub-layers (hidden
    2048, 16 heads x 128, D = 1024; random init, seed 0; x ~ N(0, 1) of [1, 65536, 2048]
    from seed 1; bf16, fp32 states): h <- h + SSSD(RMSNorm(h)); h <- h + CHAM(RMSNorm(h)).
    One sequence leaves 16 SSSD chains and one hologram: both scans run as parallel
    sequence ranges (ranges.py).  With N ranks each takes one contiguous segment of the
    sequence (strong scaling); the segment products cross the ranks in one NCCL all_gather
    per mixer and the outputs in one more.  Also times the scans alone, ranges against one
    chain (N = 1)."""
    import torch
    from verace_v1_b200.kernels import launch_cham_update, launch_sssd_scan
    from verace_v1_b200.ranges import cham_scan_ranges, pick_ranges, sssd_scan_ranges
    c = C4
    torch.manual_seed(0)
    sssd_norm = torch.nn.RMSNorm(c["hidden"], eps=1e-6)
    sssd = V.SSSDAttention(c["hidden"], c["heads"], c["head_dim"], 256)
    cham_norm = torch.nn.RMSNorm(c["hidden"], eps=1e-6)
    cham = V.ContinuousHolographicMemory(c["hidden"], c["holo"])
    mods = torch.nn.ModuleList([sssd_norm, sssd, cham_norm, cham]).to(dev, torch.bfloat16).eval()
    seg = c["seq"] // world
    x = torch.randn(1, c["seq"], c["hidden"], generator=torch.Generator().manual_seed(1))
    xs = x[:, rank * seg:(rank + 1) * seg].to(dev, torch.bfloat16)
    del x
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    Rs = pick_ranges(c["heads"], seg, dev, per_sm=1)
    Rc = pick_ranges(c["holo"] // 32, seg, dev, per_sm=2)

    def step():
        h = xs.clone()
        n = V.rmsnorm(h, sssd_norm)
        q, k, v, dl = sssd.project(n)
        if group is None:
            o, _ = launch_sssd_scan(q, k, v, dl)
        else:
            o, _ = sssd_scan_ranges(q, k, v, dl, None, Rs, group)
        n = V.add_rmsnorm(h, sssd.finish(o), out_norm=cham_norm)
        q, k, v, g = cham.project(n)
        if group is None:
            rec, _ = launch_cham_update(q, k, v, g)
        else:
            rec, _ = cham_scan_ranges(q, k, v, g, None, Rc, group)
        V.add_rmsnorm(h, cham.w_out(rec), y_norm=cham.norm)
        return gather_outputs(world, h)

    def timed(fn, reps):
        fn()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / reps)

    with torch.no_grad():
        ms = timed(step, 3)
        res = {"workload": "config 4: one SSSD + CHAM layer, b=1 x s=65536, hidden 2048, 16x128 heads, D=1024, "
                           "bf16; the scans as parallel sequence ranges"
                           + (f"; the sequence split over {world} ranks (strong scaling)" if world > 1 else ""),
               "scaling": "strong", "n_gpus": world, "ms_per_step": ms,
               "token_layers_per_s": c["seq"] / (ms * 1e-3), "ranges": {"sssd": Rs, "cham": Rc}}
        if world == 1:
            n = V.rmsnorm(xs, sssd_norm)
            qs, ks, vs, dl = sssd.project(n)
            qc, kc, vc, g = cham.project(n)
            res["sssd_scan_ms"] = timed(lambda: launch_sssd_scan(qs, ks, vs, dl), 3)
            res["sssd_scan_one_chain_ms"] = timed(lambda: launch_sssd_scan(qs, ks, vs, dl, _ranges=False), 2)
            res["cham_scan_ms"] = timed(lambda: launch_cham_update(qc, kc, vc, g), 3)
            res["cham_scan_one_chain_ms"] = timed(lambda: launch_cham_update(qc, kc, vc, g, _ranges=False), 1)
            _, _, bf16_sus, _ = _peaks()
            flop = c["seq"] * (18.0 * c["heads"] * c["head_dim"] ** 2 + 18.0 * c["holo"] ** 2)
            t = (res["sssd_scan_ms"] + res["cham_scan_ms"]) * 1e-3
            res["scan_roofline"] = {"bound": "tensor", "flop": flop, "achieved": flop / t / 1e12, "peak": bf16_sus,
                                    "unit": "TFLOP/s", "frac": flop / t / 1e12 / bf16_sus,
                                    "basis": "18 h d^2 + 18 D^2 FLOP per token (necessary), both scans"}
    del mods, xs
    return res


def run_mcmoe(args, V, dev, barrier, max_over_ranks):
    """The M-CMoE sub-layer (ManifoldContinuousMoE, mcmoe.py:58-120) at the config-2 token
    count per GPU (b*s = 16384 tokens, hidden 1024, rank 32, 64 components, top-8, the
    reference config's M-CMoE), bf16, random init; inputs resident in HBM, larger than L2
    together (x 32 MB, hyper-network output 64 MB, the projection's intermediate 64 MB).
    Times the manifold projection alone (verace_mcmoe_projection: two tcgen05 GEMMs) and
    the whole sub-layer (base SiTU-GLU FFN, routing, projection, RMSNorm + residual)."""
    import torch
    c = CFG
    n, d, r, C, K = c["batch"] * c["seq"], c["hidden"], 32, 64, 8
    torch.manual_seed(0)
    m = V.ManifoldContinuousMoE(hidden_dim=d, rank=r, num_components=C, top_k_components=K).to(dev, torch.bfloat16)
    m.eval()
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(1, n, d, generator=g, device=dev).to(torch.bfloat16)
    with torch.no_grad():
        xf = x.view(n, d)
        idx, w = V.launch_mcmoe_route(m.router(xf), K)
        pre = m.hyper_sigma(xf)
        proj = lambda: V.launch_mcmoe_projection(xf, m.u_basis, m.v_basis, idx, w, pre, sigma_is_logits=True)
        full = lambda: m(x)

        def timed(fn, reps):
            for _ in range(max(args.warmup, 3)):
                fn()
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            barrier()
            return max_over_ranks(e0.elapsed_time(e1) / reps)

        p_ms = timed(proj, 20)
        f_ms = timed(full, 10)
    _, bf16_burst, _, peak_kind = _peaks()
    dense = 4.0 * n * d * C * r            # the two GEMMs over all components
    active = 4.0 * n * d * K * r           # the selected components only (the reference's count)
    tf = dense / (p_ms * 1e-3) / 1e12
    return {"workload": f"M-CMoE sub-layer, {n} tokens, hidden {d}, rank {r}, {C} components, top-{K}, bf16",
            "projection_us": p_ms * 1e3, "sublayer_us": f_ms * 1e3,
            "tokens_per_s": n / (f_ms * 1e-3),
            "roofline": {"kernel": "mcmoe_gemm_kernel x2 (verace_mcmoe_projection)", "bound": "tensor",
                         "achieved": tf, "peak": bf16_burst, "unit": "TFLOP/s", "frac": tf / bf16_burst,
                         "flop_per_call": dense, "active_flop_per_call": active,
                         "peak_source": f"{peak_kind} bf16 dense GEMM (MEASURED_PEAKS.json, burst)"}}


def run_decode(args, layers, embed, V, dev, rank, barrier, max_over_ranks):
    """Config 3: prefill a prompt, then time single-token decode steps (CUDA graphs)."""
    import torch
    from verace_v1_b200 import _lib
    from verace_v1_b200.kernels import launch_cham_update
    c = CFG
    b, P, n = DEC["batch"], DEC["prompt"], DEC["steps"]
    nh, d, D = c["heads"], c["head_dim"], c["holo"]
    nl = len(layers)
    gen = torch.Generator().manual_seed(100 + rank)
    prompt = torch.randint(0, c["vocab"], (b, P), generator=gen).to(dev)
    toks = torch.randint(0, c["vocab"], (b, n + args.warmup), generator=gen).to(dev)
    st = V.DecodeState(nl, b, nh, d, D, device=dev, pending_depth=DEC["pending"])
    with torch.no_grad():
        x = embed(prompt).contiguous()
        nrm = V.rmsnorm(x, layers[0]["sssd_norm"])
        for l, L in enumerate(layers):
            o, psi = L["sssd"](nrm, return_state=True)
            nrm = V.add_rmsnorm(x, o, out_norm=L["cham_norm"])
            cm = L["cham"]
            q, k, v, g = cm.project(nrm)
            rec, holo = launch_cham_update(q, k, v, g)
            nxt = layers[l + 1]["sssd_norm"] if l + 1 < nl else None
            nrm = V.add_rmsnorm(x, cm.w_out(rec), y_norm=cm.norm, out_norm=nxt)
            st.load_layer(l, psi, holo)
            del o, psi, q, k, v, g, rec, holo
        del x, nrm
        saved = (st.psi.clone(), st.H_real.clone(), st.H_imag.clone())
        torch.cuda.empty_cache()
        tok = torch.zeros(b, dtype=torch.long, device=dev)

        def dstep():
            hcur = embed(tok).unsqueeze(1).contiguous()
            nrm = V.rmsnorm(hcur, layers[0]["sssd_norm"])
            for l, L in enumerate(layers):
                sm, cm = L["sssd"], L["cham"]
                q, k, v, dl = sm.project(nrm)
                o = st.step_sssd(l, q, k, v, dl)
                nrm = V.add_rmsnorm(hcur, sm.finish(o.view(b, 1, nh, d)), out_norm=L["cham_norm"])
                # the projection epilogue inside the deferred step's first kernel
                rec = st.step_cham_projected(l, cm.projection(nrm))
                nxt = layers[l + 1]["sssd_norm"] if l + 1 < nl else None
                nrm = V.add_rmsnorm(hcur, cm.w_out(rec.view(b, 1, D)), y_norm=cm.norm, out_norm=nxt)
            return hcur

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                dstep()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        l0 = _lib.lib().verace_kernel_launches()
        with torch.cuda.graph(graph):
            dstep()
        launches_per_step = int(_lib.lib().verace_kernel_launches() - l0)

        def restore():
            st.psi.copy_(saved[0])
            st.H_real.copy_(saved[1])
            st.H_imag.copy_(saved[2])
            if st.P > 0:
                st.pending.zero_()

        for i in range(args.warmup):
            tok.copy_(toks[:, n + i])
            graph.replay()
        restore()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            tok.copy_(toks[:, i])
            graph.replay()
        e1.record()
        barrier()
        us_step = max_over_ranks(e0.elapsed_time(e1)) * 1e3 / n
        if V.device_status(dev) != 0:
            raise RuntimeError("decode steps reported a device status")

        # the dominant kernel alone: the CHAM decode step (deferred updates: one read pass
        # over the hologram per step, the pending factors folded in every P-th step), timed
        # over P steps per layer so that each layer folds once
        g1 = torch.Generator().manual_seed(7)
        nrm = torch.nn.functional.normalize
        cq, ck, cv = (nrm(torch.randn(b, D, generator=g1), dim=-1).to(dev, torch.bfloat16) for _ in range(3))
        cg = (0.1 * torch.sigmoid(torch.randn(b, generator=g1))).to(dev)
        for l in range(nl):
            st.step_cham(l, cq, ck, cv, cg)
        torch.cuda.synchronize()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        reps = max(st.P, 1)
        e2.record()
        for _ in range(reps):
            for l in range(nl):
                st.step_cham(l, cq, ck, cv, cg)
        e3.record()
        torch.cuda.synchronize()
        us_launch = e2.elapsed_time(e3) * 1e3 / (reps * nl)
    graph.reset()
    del graph, saved, st
    torch.cuda.empty_cache()
    hbm = _peaks()[0]
    # Hr, Hi read once per step and written once per P steps (deferred updates)
    pdepth = DEC["pending"]
    cham_bytes = 2 * b * D * D * 4 * (1 + 1 / pdepth)
    sssd_bytes = 2 * b * nh * d * d * 4
    w_bytes = sum(p.numel() * p.element_size() for L in layers for p in L.parameters())
    step_bytes = nl * (cham_bytes + sssd_bytes) + w_bytes
    achieved = cham_bytes / (us_launch * 1e-6) / 1e9
    return {
        "workload": f"config 3: 12-layer decode, b={b} per GPU, prompt {P} (prefilled by the scans), "
                    f"{n} single-token steps (teacher-forced random ids), bf16, one CUDA graph per step, "
                    f"hologram updates deferred {DEC['pending']} steps",
        "us_per_step": us_step, "us_per_token": us_step / b, "steps": n, "batch": b,
        "readout": "unitary (Re(H q); exact for unitary holograms)",
        "gpu_launches_per_step": launches_per_step,
        "step_hbm_roofline_us": step_bytes / (hbm * 1e9) * 1e6,
        "step_frac_of_hbm_roofline": step_bytes / (hbm * 1e9) * 1e6 / us_step,
        "roofline": {"kernel": "lazy_pre_kernel + lazy_cham_kernel (CHAM decode step: one read of the hologram, "
                               "the pending rank-2 factors folded in every 8th step)",
                     "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": None, "bytes_per_launch": cham_bytes,
                     "us_per_launch": us_launch},
    }


# ------------------------------------------------------------------------------ CPU arm
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_modules():
    """The reference package from its offline install under baseline/_ref (its own
    modules, unmodified), or None when it is not installed."""
    if not os.path.isdir(os.path.join(REF_DIR, "verace_v1")):
        return None
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    from verace_v1.modules.sssd_attention import SSSDAttention
    from verace_v1.modules.cham_memory import ContinuousHolographicMemory
    return SSSDAttention, ContinuousHolographicMemory


def cpu_sample(tokens=16):
    """Time the reference's CPU path for one item x `tokens` tokens through one layer's
    SSSD and CHAM (config-1 modules: hidden 1024, 8 heads x 128, D = 1024, fp32, seed 0).

    With the reference installed (baseline/_ref) this runs the reference's own eager
    modules (SSSDAttention.forward sssd_attention.py:103-182, ContinuousHolographicMemory
    .forward cham_memory.py:117-243) on CPU tensors with torch's default thread count
    ("kind": "reference"); otherwise the numpy restatement of the same algorithm in
    oracle/ ("kind": "port")."""
    import numpy as np
    c = CFG
    hid, h, d, D = c["hidden"], c["heads"], c["head_dim"], c["holo"]
    ref = _reference_modules()
    if ref is not None:
        import torch
        SSSD, CHAM = ref
        torch.manual_seed(0)
        sssd, cham = SSSD(hid, h, d, 256).eval(), CHAM(hid, D).eval()
        x = torch.randn(1, tokens, hid, generator=torch.Generator().manual_seed(0))
        with torch.no_grad():
            t0 = time.perf_counter()
            sssd(x, return_state=True)
            cham(x)
            dt = time.perf_counter() - t0
        return {"value": tokens / dt, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "reference",
                "sample": f"1 sequence x {tokens} tokens x 1 layer: the reference's eager SSSDAttention + "
                          f"ContinuousHolographicMemory (config-1 modules, D=1024, fp32, CPU, "
                          f"{torch.get_num_threads()} torch threads), {dt:.1f} s"}
    import oracle
    rng = np.random.default_rng(0)
    bound = 1.0 / np.sqrt(hid)
    u = lambda *shape: rng.uniform(-bound, bound, size=shape).astype(np.float32)
    ps = {"w_q.weight": u(h * d, hid), "w_k.weight": u(h * d, hid), "w_v.weight": u(h * d, hid),
          "w_delta.weight": u(h, hid), "head_rmsnorm.weight": np.ones(d, np.float32),
          "w_out.weight": u(hid, h * d).astype(np.float32)}
    pc = {"w_q.weight": u(D, hid), "w_k.weight": u(D, hid), "w_v.weight": u(D, hid),
          "w_gamma.weight": u(1, hid), "w_out.weight": (rng.uniform(-1, 1, (hid, D)) / np.sqrt(D)).astype(np.float32),
          "norm.weight": np.ones(hid, np.float32)}
    x = rng.standard_normal((1, tokens, hid)).astype(np.float32)
    t0 = time.perf_counter()
    oracle.sssd_forward(ps, x, h, d, return_state=True, dtype=np.float32)
    oracle.cham_forward(pc, x, dtype=np.float32)
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 sequence x {tokens} tokens x 1 layer (SSSD + CHAM, D=1024, fp32, numpy "
                      f"eager restatement), {dt:.1f} s"}


def run_triton_bar(dev, steps=2):
    """The reference's own GPU decode path, timed on this GPU: its Triton launchers
    (launch_sssd_triton_scan, triton_kernels.py:603-636; launch_cham_triton_update, which at
    D = 1024 takes the host-looped tiled path launch_cham_triton_tiled, :552-597), unmodified
    from the offline install under baseline/_ref, for ONE layer of a config-3 decode step:
    b = 64 items, one token each, carried states (8 heads x 128, D = 1024), bf16 inputs.
    One warm-up step (Triton JIT), then `steps` timed steps with CUDA events; the full
    12-layer step is 12 x this (the projections and glue around the mixers not counted)."""
    import torch
    if not os.path.isdir(os.path.join(REF_DIR, "verace_v1")):
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    try:
        from verace_v1.serving import triton_kernels as TK
    except Exception as e:        # noqa: BLE001 -- report why the bar could not be taken
        return {"unavailable": f"reference Triton kernels not importable: {e!r}"[:300]}
    b, h, d, D = DEC["batch"], CFG["heads"], CFG["head_dim"], CFG["holo"]
    g = torch.Generator(device=dev).manual_seed(11)
    nrm = torch.nn.functional.normalize
    rn = lambda *sh: torch.randn(*sh, generator=g, device=dev)
    sq, sk, sv = (nrm(rn(b, 1, h, d), dim=-1).to(torch.bfloat16) for _ in range(3))
    dl = 0.1 * torch.sigmoid(rn(b, 1, h))
    cq, ck, cv = (nrm(rn(b, 1, D), dim=-1).to(torch.bfloat16) for _ in range(3))
    gm = 0.1 * torch.sigmoid(rn(b, 1))
    psi = torch.eye(d, device=dev).expand(b, h, d, d).contiguous()
    holo = (torch.eye(D, device=dev).expand(b, D, D).contiguous(), torch.zeros(b, D, D, device=dev))

    def step(psi, holo):
        _, psi = TK.launch_sssd_triton_scan(sq, sk, sv, dl, psi)
        _, holo = TK.launch_cham_triton_update(cq, ck, cv, gm, holo)
        return psi, holo

    with torch.no_grad():
        psi, holo = step(psi, holo)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(steps):
            psi, holo = step(psi, holo)
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    us = e0.elapsed_time(e1) * 1e3 / steps
    return {"workload": f"reference Triton decode, one layer: b={b}, 1 token per item, carried states, "
                        f"{h}x{d} heads, D={D}, bf16 inputs (baseline/_ref, unmodified)",
            "us_per_layer_step": us, "us_per_step_12_layers_extrapolated": 12 * us,
            "us_per_token_12_layers_extrapolated": 12 * us / b, "steps_timed": steps,
            "host_wall_s": wall}


def run_triton_c1(V, dev):
    """Config 1's two mixer scans (b = 2, s = 512, 8 x 128 heads, D = 1024, fp32) through the
    reference's own Triton launchers (baseline/_ref, unmodified; at D = 1024 CHAM takes the
    host-looped tiled path, triton_kernels.py:552-597) and through this package's launchers,
    on the same inputs, one timed call each after a warm-up (the reference's on a 2-token
    prefix, for its JIT); CUDA events on the current stream."""
    import torch
    if not os.path.isdir(os.path.join(REF_DIR, "verace_v1")):
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    try:
        from verace_v1.serving import triton_kernels as TK
    except Exception as e:        # noqa: BLE001 -- report why the timing could not be taken
        return {"unavailable": f"reference Triton kernels not importable: {e!r}"[:300]}
    b, s, h, d, D = 2, 512, CFG["heads"], CFG["head_dim"], CFG["holo"]
    g = torch.Generator(device=dev).manual_seed(12)
    nrm = torch.nn.functional.normalize
    rn = lambda *sh: torch.randn(*sh, generator=g, device=dev)
    sq, sk, sv = (nrm(rn(b, s, h, d), dim=-1) for _ in range(3))
    dl = 0.1 * torch.sigmoid(rn(b, s, h))
    cq, ck, cv = (nrm(rn(b, s, D), dim=-1) for _ in range(3))
    gm = 0.1 * torch.sigmoid(rn(b, s))

    def timed(fn):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1), out

    with torch.no_grad():
        TK.launch_sssd_triton_scan(sq[:, :2], sk[:, :2], sv[:, :2], dl[:, :2])
        TK.launch_cham_triton_update(cq[:, :2], ck[:, :2], cv[:, :2], gm[:, :2])
        ref_ms, (ro_s, ro_c) = timed(lambda: (TK.launch_sssd_triton_scan(sq, sk, sv, dl)[0],
                                              TK.launch_cham_triton_update(cq, ck, cv, gm)[0]))
        V.launch_sssd_scan(sq, sk, sv, dl)
        V.launch_cham_update(cq, ck, cv, gm)
        ours_ms, (oo_s, oo_c) = timed(lambda: (V.launch_sssd_scan(sq, sk, sv, dl)[0],
                                               V.launch_cham_update(cq, ck, cv, gm)[0]))
    rel = lambda a, r: float((a.float() - r.float()).norm() / r.float().norm())
    return {"workload": f"config 1's mixer scans: SSSD ({h}x{d}) + CHAM (D={D}) over b={b} x s={s}, fp32 "
                        "inputs, no initial state",
            "reference_triton_ms": ref_ms, "ours_ms": ours_ms, "ratio": ref_ms / ours_ms,
            "rel_diff_sssd_out": rel(oo_s, ro_s), "rel_diff_cham_out": rel(oo_c, ro_c)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_sample(tokens=args.ref_tokens)
    t0 = time.perf_counter()
    vals = [cpu_sample(tokens=args.ref_tokens) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    value = args.ref_tokens * args.steps / wall
    ms = wall * 1e3 / args.steps
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "config 2's per-layer mixers (hidden 1024, 8x128 heads, D=1024) on a bounded CPU "
                               f"sample: 1 sequence x {args.ref_tokens} tokens x 1 layer per step",
                   "global_batch": 1, "seq_len": args.ref_tokens, "layers": 1,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": vals[-1]["cores"], "kind": vals[-1]["kind"],
                         "sample": vals[-1]["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_only(args):
    """Kernel-level case used for profiling: one scan entry point on synthetic inputs."""
    import torch
    _load_package()
    from verace_v1_b200.kernels import launch_cham_update, launch_sssd_scan
    c = CFG
    dev = torch.device("cuda", 0)
    b, s = args.batch or c["batch"], args.seq or c["seq"]
    g = torch.Generator().manual_seed(0)
    nrm = torch.nn.functional.normalize
    if args.only == "mcmoe":
        V = sys.modules["verace_v1_b200"]
        n, d, r, C, K = b * s, c["hidden"], 32, 64, 8
        torch.manual_seed(0)
        m = V.ManifoldContinuousMoE(hidden_dim=d, rank=r, num_components=C, top_k_components=K)
        m = m.to(dev, torch.bfloat16).eval()
        xf = torch.randn(n, d, generator=g).to(dev, torch.bfloat16)
        with torch.no_grad():
            idx, w = V.launch_mcmoe_route(m.router(xf), K)
            pre = m.hyper_sigma(xf)
        fn = lambda: V.launch_mcmoe_projection(xf, m.u_basis, m.v_basis, idx, w, pre, sigma_is_logits=True)
    elif args.only == "decode":
        V = sys.modules["verace_v1_b200"]
        D = c["holo"]
        st = V.DecodeState(1, b, c["heads"], c["head_dim"], D, device=dev)
        q, k, v = (nrm(torch.randn(b, D, generator=g), dim=-1).to(dev, torch.bfloat16) for _ in range(3))
        gam = (0.1 * torch.sigmoid(torch.randn(b, generator=g))).to(dev)
        fn = lambda: st.step_cham(0, q, k, v, gam)
    elif args.only == "decode_step":   # the whole config-3 decode leg (12 layers, CUDA graph per step)
        V = sys.modules["verace_v1_b200"]
        layers, embed = build_chain(V, dev)
        res = run_decode(args, layers, embed, V, dev, 0, torch.cuda.synchronize, lambda x: x)
        print(json.dumps({"only": args.only, **res}), flush=True)
        return
    elif args.only == "retract":
        V = sys.modules["verace_v1_b200"]
        D = c["holo"]
        Hr = (torch.eye(D).expand(b, D, D) + 0.01 * torch.randn(b, D, D, generator=g)).to(dev)
        Hi = (0.01 * torch.randn(b, D, D, generator=g)).to(dev)
        fn = lambda: V.newton_schulz_unitary_retraction(Hr, Hi, 3)
    elif args.only == "cham":
        D = c["holo"]
        q, k, v = (nrm(torch.randn(b, s, D, generator=g), dim=-1).to(dev, torch.bfloat16) for _ in range(3))
        gam = (0.1 * torch.sigmoid(torch.randn(b, s, generator=g))).to(dev)
        fn = lambda: launch_cham_update(q, k, v, gam)
    else:
        h, d = c["heads"], c["head_dim"]
        q, k, v = (nrm(torch.randn(b, s, h, d, generator=g), dim=-1).to(dev, torch.bfloat16) for _ in range(3))
        dl = (0.1 * torch.sigmoid(torch.randn(b, s, h, generator=g))).to(dev)
        fn = lambda: launch_sssd_scan(q, k, v, dl)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"only": args.only, "batch": b, "seq": s, "ms_per_call": ms,
                      "tokens_per_s": b * s / (ms * 1e-3)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-tokens", type=int, default=32)
    ap.add_argument("--ref-tokens", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-3 decode measurement")
    ap.add_argument("--no-mcmoe", action="store_true", help="skip the M-CMoE sub-layer measurement")
    ap.add_argument("--no-long", action="store_true", help="skip the config-4 long-sequence measurement")
    ap.add_argument("--no-model", action="store_true", help="skip the whole-model config-2 prefill measurement")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the config-5 one-layer strong-scaling measurement")
    ap.add_argument("--no-triton-bar", action="store_true",
                    help="skip timing the reference's Triton decode path (one layer, config 3)")
    ap.add_argument("--only", choices=["cham", "sssd", "decode", "decode_step", "mcmoe", "retract"], default=None,
                    help="time one scan entry point alone (kernel-level case for profiling)")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    args = ap.parse_args()
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
