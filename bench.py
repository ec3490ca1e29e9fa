#!/usr/bin/env python
"""Benchmark of the Q4 decode path on B200 — prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload (the metric's decode tokens/s): one greedy decode step = 24 x [RMSNorm
(1+w) -> Q4 SwiGLU MLP 2048<->6144 -> residual] -> final RMSNorm -> Q4 lm_head 248320x2048 -> argmax,
seeded synthetic weights (N(0,0.02) via the seeded generator) and embeddings (N(0,1)), batch B
(default 1).  At N > 1 the step is tensor-parallel (column/row-split MLP, vocabulary-sharded
lm_head): the per-layer all-reduce and the argmax merge run inside the kernels over NVLink peer
memory (marlin_q4_tp_decode_step): strong scaling.

`value` is tokens/s of the whole job: CUDA events around K CUDA-graph replays (weights stream
795.7 MB per step, > 126 MB L2: every step reads HBM), the K-step measurement repeated until at
least one second has been timed, each repeat bracketed by a barrier and a synchronize, the max over
ranks per repeat, the median over repeats.  `e2e` repeats the measurement through the public API
with the step's embeddings copied from pinned host memory and the token ids read back to the host
every step (on one GPU through `marlin_q4.HostDecodeStep`: the two copies and the step replayed as
one CUDA graph, then a synchronisation; at N > 1 the copies run as stream operations around the
step's graph).  `roofline` covers the step's dominant part, the MLP layers as they run inside the step
(at N = 1 one persistent kernel for all layers, at N > 1 two kernels per layer; per-layer time =
(t(24 layers) - t(1 layer)) / 23, both CUDA-graph replays of the same public call; per rank at
N > 1).  `extras.step_per_layer_kernels` times the N = 1 step on the per-layer kernels as well.  At N > 1 `parity` compares the sharded step's ids and h
with the unsharded single-GPU step on the same inputs; `extras.batch_sweep` gives batch 1/8/32 and
`extras.prefill_c4` the config-4 prefill MLP layer at every N.  `gemv` is the metric's first half
(config 1: one 6144x2048 Q4 GEMV, bf16 x, N = 1).

--impl reference times the CPU restatement of the reference's Q4 path (oracle/, OpenMP on all host
threads) on the same workload: MLX, which holds the reference's arithmetic, is absent here.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "marlin-mlx_b200"))

H, I, V, L = 2048, 6144, 248320, 24
Q4_MAT = 7_077_888               # bytes of one 2048x6144 / 6144x2048 Q4 matrix (packed + scales + biases)
LM_BYTES = 286_064_640           # 248320x2048 Q4
STEP_WEIGHT_BYTES = 795_672_576  # 24 x 3 x Q4_MAT + LM_BYTES


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bound on the CPU baseline sample")
    ap.add_argument("--no-extras", action="store_true", help="skip the per-family and batch sweeps")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg (profiling runs)")
    ap.add_argument("--min-seconds", type=float, default=1.0, help="repeat the K-step timing until this much is timed")
    return ap.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------------------------
# clocks sampler (nvidia-smi, 200 ms) during the timed region
# ---------------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# model construction (seeded; same seeds for every N so TP shards the same model)
# ---------------------------------------------------------------------------------------------
def build_model(mq, tp_rank: int, tp: int):
    import torch
    from marlin_q4 import tp as tpmod
    layers = []
    for l in range(L):
        g = mq.quantize_weight(mq.synth_bf16((I, H), 1000 + 4 * l, 0.0, 0.02))
        u = mq.quantize_weight(mq.synth_bf16((I, H), 1001 + 4 * l, 0.0, 0.02))
        d = mq.quantize_weight(mq.synth_bf16((H, I), 1002 + 4 * l, 0.0, 0.02))
        nw = mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02)
        layer = mq.Layer(nw, g, u, d)
        layers.append(tpmod.shard_layer(layer, tp_rank, tp, k_multiple=512) if tp > 1 else layer)
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 2000, 0.0, 0.02))
    off = 0
    if tp > 1:
        lm, off = tpmod.shard_vocab(lm, tp_rank, tp)
    torch.cuda.empty_cache()
    fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
    return layers, fn, lm, off


METRIC = "Q4 MLP+lm_head decode tokens/s (24-layer Q4 SwiGLU MLP stack + Q4 lm_head + argmax)"


def config_dict(B: int, world: int) -> dict:
    """The workload both arms report (identical keys and values for the same batch and N)."""
    return {"workload": "C5 decode step: 24 x [RMSNorm(1+w) -> Q4 SwiGLU MLP 2048<->6144 -> residual] + "
                        "final RMSNorm + Q4 lm_head 248320x2048 + argmax",
            "batch": B, "tp": world, "layers": L, "hidden": H, "intermediate": I, "vocab": V,
            "weight_bytes_per_step": STEP_WEIGHT_BYTES,
            "l2": "no flush: 795.7 MB of weights per step > 126 MB L2",
            "parallelism": f"tp{world}" if world > 1 else "single"}


def max_over_ranks(torch, dist, values, dev):
    """Elementwise max over ranks of a list of floats (identity at N = 1)."""
    if not dist.is_initialized():
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def capture(torch, fn):
    """fn() captured in a CUDA graph (after one eager call on a side stream)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_graph(torch, fn, reps: int, warm: int = 3) -> float:
    """Capture fn() in a CUDA graph; return ms per replay over `reps` replays (CUDA events).  Every
    rank of a multi-GPU run calls it with the same arguments (the replays exchange data)."""
    g = capture(torch, fn)
    for _ in range(warm):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / reps
    del g
    return ms


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    import marlin_q4 as mq
    from marlin_q4 import tp as tpmod

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"  # no version banner on stdout: the JSON line stays alone there
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    B = args.batch
    layers, fn, lm, off = build_model(mq, rank, world)
    h0 = mq.synth_bf16((B, H), 3000, 0.0, 1.0)

    def make_step(lys, m):
        # at N > 1 the exchanges run inside the kernels over NVLink peer memory (no collective call per step)
        return tpmod.FusedTPDecodeStep(lys, fn, lm, off, m) if world > 1 else mq.DecodeStep(lys, fn, lm, m)

    def close(st):
        if world > 1:
            st.close()

    step = make_step(layers, B)
    graph = capture(torch, lambda: step(h0))
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    barrier()

    # timed region: K replays per repeat, repeated until >= min_seconds (max over ranks per repeat)
    def one_repeat() -> float:
        barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            graph.replay()
        t1.record()
        torch.cuda.synchronize()
        barrier()
        return t0.elapsed_time(t1)

    clocks = Clocks(local)
    clocks.start()
    first = max_over_ranks(torch, dist, [one_repeat()], dev)[0]
    repeats = int(min(2000, max(1, -(-args.min_seconds * 1e3 // max(first, 1e-3)))))
    rep_ms = [one_repeat() for _ in range(repeats)]
    ck = clocks.stop()
    rep_ms = max_over_ranks(torch, dist, rep_ms, dev)
    rep_ms.sort()
    ms = statistics.median(rep_ms) / args.steps
    value = B / (ms / 1e3)
    dist_ms = {"repeats": repeats, "steps_per_repeat": args.steps,
               "timed_s": round(sum(rep_ms) / 1e3, 3),
               "p10": round(rep_ms[len(rep_ms) // 10] / args.steps, 5),
               "p50": round(ms, 5),
               "p90": round(rep_ms[min(len(rep_ms) - 1, (9 * len(rep_ms)) // 10)] / args.steps, 5)}

    # e2e: public API with host buffers (H2D of embeddings, D2H of ids every step)
    h_host = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()
    h_host.copy_(h0.cpu())
    ids_host = torch.empty(B, dtype=torch.int32).pin_memory()
    if world == 1:
        # marlin_q4.HostDecodeStep: the copy in, the step and the copy out as one graph per token
        host_step = mq.HostDecodeStep(step, h_host, ids_host)
    else:
        # tensor-parallel step: the copies as stream operations around the step's graph
        def host_step():
            h0.copy_(h_host, non_blocking=True)
            graph.replay()
            ids_host.copy_(step.ids, non_blocking=True)
            torch.cuda.current_stream().synchronize()
    for _ in range(3):
        host_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        host_step()  # H2D of the embeddings, the step, D2H of the ids, then the host waits for them
    e1.record()
    e1.synchronize()
    e2e_ms = max_over_ranks(torch, dist, [e0.elapsed_time(e1) / args.steps], dev)[0]
    if world == 1:
        host_step.close()
    ids_run, h_run = step.ids.clone(), step.h.clone()
    del graph
    close(step)

    pk = peaks()
    extras, roof, gemv, parity = {}, None, None, None
    reps = max(5, args.steps // 2)
    if world > 1:
        # parity of the sharded step against the unsharded single-GPU step (rank 0, same seeds)
        full = build_model(mq, 0, 1) if rank == 0 else None
        if rank == 0:
            ref = mq.DecodeStep(full[0], full[1], full[2], B)
            rids, _, rh = ref(h0)
            torch.cuda.synchronize()
            parity = {"ids_equal": bool(torch.equal(rids, ids_run)),
                      "h_rel": float(((h_run - rh).abs().max() / rh.abs().max()).item()),
                      "reference": "marlin_q4_decode_step on one GPU with the unsharded weights, same inputs",
                      "bar": "ids bit-exact; h within 1e-5 of the row maximum"}
            del ref, full
            torch.cuda.empty_cache()
        barrier()
    if not args.no_extras:
        # the step's own kernels: per-layer time from steps of L and 1 layers (same weights, CUDA graphs)
        st1 = make_step(layers[:1], B)
        t_one = max_over_ranks(torch, dist, [time_graph(torch, lambda: st1(h0), reps)], dev)[0]
        close(st1)
        layer_ms = (ms - t_one) / (L - 1)
        lm_ms = t_one - layer_ms
        layer_bytes = (3 * Q4_MAT) // world + 2 * B * (H + I // world) * 4
        split = {"layer_us": round(layer_ms * 1e3, 3), "lm_head_us": round(lm_ms * 1e3, 3),
                 "layers_share": round(L * layer_ms / ms, 4), "lm_head_share": round(lm_ms / ms, 4),
                 "layer_gbs_per_gpu": round(layer_bytes / (layer_ms * 1e-3) / 1e9, 1),
                 "lm_head_gbs_per_gpu": round((LM_BYTES // world + B * H * 4) / (lm_ms * 1e-3) / 1e9, 1),
                 "method": "layer = (t(24-layer step) - t(1-layer step)) / 23, lm_head = t(1-layer step) - layer"}
        extras["step_split"] = split
        traffic = None
        tp_path = ROOT / "profiles" / "traffic.json"
        if world == 1 and B == 1 and tp_path.exists():
            traffic = json.loads(tp_path.read_text()).get("fused_layer")
        ach = layer_bytes / (layer_ms * 1e-3) / 1e9
        if world == 1:
            kname = ("fused_layers_kernel: all 24 MLP layers in one persistent launch (CTA per 64 intermediate "
                     "features, SwiGLU activations shared in 8-CTA clusters, down_proj partials in a counted "
                     "fixed-point accumulator); per layer")
            launches = 1
        else:
            kname = ("i8_unit_kernel gate/up+SwiGLU launch + i8_unit_kernel down+residual launch (cluster K split, "
                     "activation planes handed between them), per rank; the down launch's epilogue holds the "
                     "in-kernel all-reduce")
            launches = 2
        roof = {"bound": "hbm", "kernel": f"mlp_layer: {kname}, as run inside the step",
                "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(ach / pk["hbm_gbs"], 4),
                "traffic": traffic, "algorithmic_bytes_per_layer": layer_bytes, "launches_per_layer": launches,
                "layer_us": round(layer_ms * 1e3, 3), "peak_source": pk["source"],
                "share_of_step": split["layers_share"]}
        if world == 1:
            # the same step on the per-layer kernels (two cluster split-K launches per layer), for comparison
            mq.set_step_kernels("layers")
            try:
                stl = make_step(layers, B)
                t_layers = time_graph(torch, lambda: stl(h0), reps)
                del stl
            finally:
                mq.set_step_kernels("fused")
            extras["step_per_layer_kernels"] = {"ms_per_step": round(t_layers, 4),
                                                "tokens_per_s": round(B / (t_layers / 1e3), 1),
                                                "note": "marlin_q4_set_step_kernels(MARLIN_Q4_STEP_LAYERS)"}

        # batch sweep of the full step (every N)
        sweep = {}
        for bb in (1, 8, 32):
            if bb == B:
                sweep[f"batch{bb}"] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(value, 1)}
                continue
            st = make_step(layers, bb)
            hb = mq.synth_bf16((bb, H), 3001, 0.0, 1.0)
            msb = max_over_ranks(torch, dist, [time_graph(torch, lambda: st(hb), max(5, args.steps // 4))], dev)[0]
            sweep[f"batch{bb}"] = {"ms_per_step": round(msb, 4), "tokens_per_s": round(bb / (msb / 1e3), 1),
                                   "step_hbm_frac_per_gpu": round(STEP_WEIGHT_BYTES / world / (msb * 1e-3) / 1e9
                                                                  / pk["hbm_gbs"], 4)}
            close(st)
            del st
        extras["batch_sweep"] = sweep

        # config 4: prefill MLP layer, x bf16 [2048, 2048] -> gate/up + SwiGLU -> down (tcgen05 GEMMs);
        # at N > 1 over the ranks (column/row shards, NCCL all-reduce of the binary32 partials)
        xp = mq.synth_bf16((2048, H), 3002, 0.0, 1.0)
        flops = 3 * 2.0 * 2048 * I * H
        if world == 1:
            ap_ = torch.empty((2048, I), dtype=torch.bfloat16, device=dev)
            L0 = layers[0]

            def prefill_layer():
                mq.gate_up_swiglu(xp, L0.gate_proj, L0.up_proj, out=ap_)
                mq.qmatmul(ap_, L0.down_proj)
            desc = "C4: x bf16 [2048,2048] -> Q4 gate/up (SwiGLU) -> Q4 down, one layer"
        else:
            full0 = mq.Layer(*[t for t in build_layer0(mq)])
            pmlp = tpmod.TPPrefillMLP(tpmod.shard_layer(full0, rank, world, k_multiple=512, pad_gate_up=True), 2048)
            del full0

            def prefill_layer():
                pmlp(xp)
            desc = (f"C4 over {world} GPUs: gate/up row shards + SwiGLU, down K shards with binary32 partials, "
                    "NCCL all-reduce(sum), bf16 cast; one layer")
        t_pf = max_over_ranks(torch, dist, [time_graph(torch, prefill_layer, 10)], dev)[0]
        tfs = flops / (t_pf * 1e-3) / 1e12
        extras["prefill_c4"] = {"config": desc, "us_per_layer": round(t_pf * 1e3, 2), "tflops": round(tfs, 1),
                                "tflops_per_gpu": round(tfs / world, 1),
                                "frac_of_peak_burst": round(tfs / world / pk["bf16_tflops"], 4),
                                "frac_of_peak_sustained": round(tfs / world / pk["bf16_tflops_sustained"], 4),
                                "flop_per_layer": flops}

    if not args.no_extras and world == 1:
        # kernel families, each timed alone in a CUDA graph of back-to-back launches over all 24
        # layers' weights (340 MB / 170 MB > L2), PDL on — as they run inside the step
        hf = torch.empty((B, H), dtype=torch.float32, device=dev).copy_(h0.float())
        act = torch.empty((B, I), dtype=torch.float32, device=dev).normal_()
        res = torch.empty((B, H), dtype=torch.float32, device=dev)
        ws = mq.LmHeadWorkspace(B, dev)

        def fam_gateup():
            for Lr in layers:
                mq.gate_up_swiglu(hf, Lr.gate_proj, Lr.up_proj, norm_weight=Lr.post_attn_norm, out=act)

        def fam_down():
            for Lr in layers:
                mq.matmul_residual(act, Lr.down_proj, hf, out=res)

        def fam_lm():
            for _ in range(4):
                mq.lm_head_argmax(hf, lm, norm_weight=fn, workspace=ws)

        t_gu = time_graph(torch, fam_gateup, reps) / L
        t_dn = time_graph(torch, fam_down, reps) / L
        t_lm = time_graph(torch, fam_lm, reps) / 4
        fams = {
            "gate_up_swiglu": {"launches_per_step": L, "us": t_gu * 1e3,
                               "bytes": 2 * Q4_MAT + B * H * 4 + B * I * 4},
            "down_residual": {"launches_per_step": L, "us": t_dn * 1e3,
                              "bytes": Q4_MAT + B * I * 4 + 2 * B * H * 4},
            "lm_head_argmax": {"launches_per_step": 1, "us": t_lm * 1e3, "bytes": LM_BYTES + B * H * 4 + B * 4},
        }
        for f in fams.values():
            f["gbs"] = f["bytes"] / (f["us"] * 1e-6) / 1e9
            f["frac_hbm"] = f["gbs"] / pk["hbm_gbs"]
            f["share_us_per_step"] = f["us"] * f["launches_per_step"]
        extras["families"] = {k: {kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                              for k, v in fams.items()}
        extras["families_note"] = ("public single-op entry points (each stages its own activations), "
                                   "not the step's kernels; see step_split for those")
        # config 1 GEMV: 6144x2048, bf16 x [1, 2048], over 24 distinct weight copies (170 MB > L2)
        xb = mq.synth_bf16((1, H), 7, 0.0, 1.0)

        def gemv_stream():
            for Lr in layers:
                mq.qmatmul(xb, Lr.gate_proj)

        t_stream = time_graph(torch, gemv_stream, reps) / L
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        iso = []
        for _ in range(20):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            mq.qmatmul(xb, layers[0].gate_proj)
            b.record()
            b.synchronize()
            iso.append(a.elapsed_time(b))
        t_iso = statistics.median(iso)
        gb = Q4_MAT + H * 2 + I * 2
        gemv = {"config": "C1: x bf16 [1,2048] . Q4 W[6144,2048]^T -> bf16 [1,6144]", "bytes": gb,
                "stream_us": round(t_stream * 1e3, 3), "stream_gbs": round(gb / (t_stream * 1e-3) / 1e9, 1),
                "stream_frac": round(gb / (t_stream * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                "isolated_us": round(t_iso * 1e3, 3), "isolated_gbs": round(gb / (t_iso * 1e-3) / 1e9, 1),
                "isolated_frac": round(gb / (t_iso * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                "note": "stream = back-to-back launches over 24 weight copies (PDL); isolated = one launch after "
                        "a 256 MB L2 flush, launch latency included"}

    # CPU baseline: the oracle (CPU restatement) on the host cores, bounded sample, rank 0 at N=1
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        cpu = cpu_baseline_from_device(layers, fn, lm, h0, B, args.cpu_seconds)

    chunks = -(-B // 8)  # above 8 rows the step runs in 8-row chunks
    # per chunk: one layer-stack launch and the lm_head at N = 1; gate/up and down per layer, then the
    # lm_head, at N > 1
    launches = args.steps * chunks * (2 if world == 1 else 2 * L + 1)
    line = {
        "metric": METRIC,
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "ms_per_step_repeats": dist_ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "q4g64 weights; u8 x s8 -> s32 tensor-core MMA on the raw codes (odd nibbles as 16q) against 4 "
                 "exact s8 activation planes per row, binary32 scale/bias fold (activations binary32 after the first "
                 "RMSNorm)",
        "data": "synthetic (seeded generator: weights N(0,0.02), norms N(0.1,0.02), embeddings N(0,1))",
        "config": config_dict(B, world),
        "clocks": ck,
        "e2e": {"value": round(B / (e2e_ms / 1e3), 2), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * 4,
                "path": ("public API marlin_q4.HostDecodeStep (pinned host embeddings in, the step, token ids out, "
                         "replayed as one CUDA graph) every step, host sync per token" if world == 1 else
                         "public API (CUDA graph of the TP step) with pinned host embeddings in and token ids out "
                         "every step as stream copies, host sync per token")},
        "gpu_launches": launches,
        "roofline": roof,
        "parity": parity,
        "gemv": gemv,
        "cpu_baseline": cpu,
        "step_hbm": {"gbs_per_gpu": round(STEP_WEIGHT_BYTES / world / (ms * 1e-3) / 1e9, 1),
                     "frac": round(STEP_WEIGHT_BYTES / world / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)},
    }
    if extras:
        line["extras"] = extras
    if world > 1:
        barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def build_layer0(mq):
    """Layer 0 of the model, unsharded (same seeds as build_model)."""
    g = mq.quantize_weight(mq.synth_bf16((I, H), 1000, 0.0, 0.02))
    u = mq.quantize_weight(mq.synth_bf16((I, H), 1001, 0.0, 0.02))
    d = mq.quantize_weight(mq.synth_bf16((H, I), 1002, 0.0, 0.02))
    nw = mq.synth_bf16((H,), 1003, 0.1, 0.02)
    return nw, g, u, d


def cpu_baseline_from_device(layers, fn, lm, h0, B, seconds):
    """Time the oracle's decode step on the host (all OpenMP threads) for a bounded number of steps."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "oracle"))
    import q4_oracle as qo
    import torch

    def u16(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    def hq(q):
        return qo.Q4(q.weight.cpu().numpy().view(np.uint32), u16(q.scales), u16(q.biases))

    C = qo.COracle()
    hl = [(u16(Lr.post_attn_norm), hq(Lr.gate_proj), hq(Lr.up_proj), hq(Lr.down_proj)) for Lr in layers]
    hlm, hfn, hh0 = hq(lm), u16(fn), u16(h0)
    C.decode_step(hh0, hl, hfn, hlm)  # warm-up (page in)
    n, t0 = 0, time.perf_counter()
    while True:
        C.decode_step(hh0, hl, hfn, hlm)
        n += 1
        if time.perf_counter() - t0 > seconds or n >= 50:
            break
    dt = time.perf_counter() - t0
    return {"value": round(B * n / dt, 3), "unit": "tokens/s", "cores": C.num_threads(), "kind": "port",
            "sample": f"{n} full decode steps (24 layers + lm_head) at batch {B}, {dt:.1f} s",
            "label": "CPU restatement of the reference's Q4 path (oracle/q4_oracle.c, OpenMP), not MLX"}


# ---------------------------------------------------------------------------------------------
# reference arm: the CPU restatement on host cores
# ---------------------------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import numpy as np
    sys.path.insert(0, str(ROOT / "oracle"))
    import q4_oracle as qo
    C = qo.COracle()
    B = args.batch
    layers = []
    for l in range(L):
        g = C.quantize(C.synth_bf16((I, H), 1000 + 4 * l, 0.0, 0.02))
        u = C.quantize(C.synth_bf16((I, H), 1001 + 4 * l, 0.0, 0.02))
        d = C.quantize(C.synth_bf16((H, I), 1002 + 4 * l, 0.0, 0.02))
        layers.append((C.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02), g, u, d))
    lm = C.quantize(C.synth_bf16((V, H), 2000, 0.0, 0.02))
    fn = C.synth_bf16((H,), 2001, 0.1, 0.02)
    h0 = C.synth_bf16((B, H), 3000, 0.0, 1.0)
    for _ in range(args.warmup):
        C.decode_step(h0, layers, fn, lm)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        C.decode_step(h0, layers, fn, lm)
    dt = time.perf_counter() - t0
    ms = dt / args.steps * 1e3
    val = B / (ms / 1e3)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(val, 4), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 (CPU)", "data": "synthetic (same seeded generator and seeds as our arm)",
        "config": config_dict(B, world),
        "cpu_baseline": {"value": round(val, 4), "unit": "tokens/s", "cores": C.num_threads(), "kind": "port",
                         "sample": f"{args.steps} full decode steps at batch {B} after {args.warmup} warm-up"},
        "e2e": {"value": round(val, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX v0.25.2 (the reference's arithmetic) cannot be built here; this arm is the CPU "
                "restatement oracle/q4_oracle.c on all host threads",
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
