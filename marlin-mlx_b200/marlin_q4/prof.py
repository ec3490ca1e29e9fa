"""Standalone driver of the decode kernels, for profilers (ncu) and quick timing.

    python -m marlin_q4.prof [--m 1] [--reps 3] [--time] [--path i8|bf16]
    python -m marlin_q4.prof --step 24 [--m 1] [--reps 3] [--time] [--path ...]

Builds one decode layer (gate/up/down Q4 [6144,2048]/[2048,6144]) and the Q4 lm_head
[248320, 2048] from the seeded generator, then launches, in this order, `reps` times each:
gate_up_swiglu (RMSNorm fused), matmul_residual (down + residual), lm_head_argmax (final norm
fused), and qmatmul (config 1: bf16 x [1, 2048] . W[6144, 2048]^T).  About 1.6 GB on the device.
With --time, prints each family's CUDA-event time per launch: `reps` launches captured in one CUDA
graph (so host launch cost is excluded), replayed after a warm-up replay.
With --step N, builds N distinct decode layers plus the lm_head and runs the whole decode step
(marlin_q4.DecodeStep) `reps` times instead (about 0.8 GB on the device for N = 24).
"""
from __future__ import annotations

import argparse

import torch

import marlin_q4 as mq

H, I, V = 2048, 6144, 248320


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--path", default="i8", choices=sorted(mq.ops.DECODE_PATHS))
    ap.add_argument("--prefill", type=int, default=0, help="time the C4 prefill layer with this many bf16 rows")
    ap.add_argument("--step", type=int, default=0, help="run the decode step of this many layers")
    a = ap.parse_args()
    torch.cuda.set_device(0)
    mq.set_decode_path(a.path)
    if a.prefill:
        prefill(a)
        return
    if a.step:
        step(a)
        return
    g = mq.quantize_weight(mq.synth_bf16((I, H), 1000, 0.0, 0.02))
    u = mq.quantize_weight(mq.synth_bf16((I, H), 1001, 0.0, 0.02))
    d = mq.quantize_weight(mq.synth_bf16((H, I), 1002, 0.0, 0.02))
    nw = mq.synth_bf16((H,), 1003, 0.1, 0.02)
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 2000, 0.0, 0.02))
    torch.cuda.empty_cache()
    fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
    h = mq.synth_bf16((a.m, H), 3000, 0.0, 1.0).float()
    act = torch.empty((a.m, I), dtype=torch.float32, device="cuda")
    res = torch.empty((a.m, H), dtype=torch.float32, device="cuda")
    xb = mq.synth_bf16((1, H), 7, 0.0, 1.0)
    ws = mq.LmHeadWorkspace(a.m, "cuda")
    fams = {
        "gate_up_swiglu": lambda: mq.gate_up_swiglu(h, g, u, norm_weight=nw, out=act),
        "down_residual": lambda: mq.matmul_residual(act, d, h, out=res),
        "lm_head_argmax": lambda: mq.lm_head_argmax(h, lm, norm_weight=fn, workspace=ws),
        "qmatmul_c1": lambda: mq.qmatmul(xb, g),
    }
    for name, f in fams.items():
        if a.time:
            f()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(a.reps):
                    f()
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            print(f"{name}: {e0.elapsed_time(e1) / a.reps * 1e3:.2f} us/launch")
            del graph
        else:
            for _ in range(a.reps):
                f()
    torch.cuda.synchronize()
    assert mq.device_error() == 0


def step(a) -> None:
    """The decode step (C5 shapes) over `a.step` distinct layers, eager launches or one CUDA graph."""
    layers = []
    for l in range(a.step):
        g = mq.quantize_weight(mq.synth_bf16((I, H), 1000 + 4 * l, 0.0, 0.02))
        u = mq.quantize_weight(mq.synth_bf16((I, H), 1001 + 4 * l, 0.0, 0.02))
        d = mq.quantize_weight(mq.synth_bf16((H, I), 1002 + 4 * l, 0.0, 0.02))
        layers.append(mq.Layer(mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02), g, u, d))
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 2000, 0.0, 0.02))
    fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
    torch.cuda.empty_cache()
    h0 = mq.synth_bf16((a.m, H), 3000, 0.0, 1.0)
    run = mq.DecodeStep(layers, fn, lm, a.m)
    if a.time:
        run(h0)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(a.reps):
                run(h0)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        print(f"decode step ({a.step} layers, m={a.m}, {a.path}): {e0.elapsed_time(e1) / a.reps * 1e3:.2f} us/step")
        del graph
    else:
        for _ in range(a.reps):
            run(h0)
    torch.cuda.synchronize()
    assert mq.device_error() == 0


def prefill(a) -> None:
    """C4: x bf16 [m, 2048] -> gate/up + SwiGLU -> down, each Q4 GEMM on the tcgen05 path."""
    g = mq.quantize_weight(mq.synth_bf16((I, H), 1000, 0.0, 0.02))
    u = mq.quantize_weight(mq.synth_bf16((I, H), 1001, 0.0, 0.02))
    d = mq.quantize_weight(mq.synth_bf16((H, I), 1002, 0.0, 0.02))
    x = mq.synth_bf16((a.prefill, H), 3000, 0.0, 1.0)
    act = torch.empty((a.prefill, I), dtype=torch.bfloat16, device="cuda")
    fams = {"gate_up_swiglu": (lambda: mq.gate_up_swiglu(x, g, u, out=act), 2 * 2.0 * a.prefill * I * H),
            "down": (lambda: mq.qmatmul(act, d), 2.0 * a.prefill * I * H)}
    for name, (f, flops) in fams.items():
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.reps):
            f()
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) / a.reps * 1e3
        print(f"{name}: {us:.2f} us/launch, {flops / us / 1e6:.1f} TFLOP/s")
    torch.cuda.synchronize()
    assert mq.device_error() == 0


if __name__ == "__main__":
    main()
