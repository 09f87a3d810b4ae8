"""Same-box comparator: the reference's own Triton kernels, timed on this GPU.

    python baseline/triton_ref.py --config cfg2 --steps 10 --warmup 3 --out RESULT.json

Imports the UNMODIFIED reference package from baseline/_ref (see
baseline/install_ref.py) and times its public entry point
``co_alibi_attention(q, k, v, causal=...)`` -- its stock code path: GQA through
``repeat_interleave``, the autotuned Triton forward, the Triton backward with its
dk/dv partial buffers -- on the same seeded inputs bench.py uses.  Three numbers,
with CUDA events on the current stream:

* forward alone (as co_alibi_attn/benchmark_flops.py:54-64 times it);
* backward alone, replaying ``backward(dout, retain_graph=True)`` on one forward
  graph with the gradients zeroed every repetition (benchmark_flops.py:66-92);
* forward + backward, a fresh graph each step (the metric bench.py reports).

The first call autotunes the forward over its ten configurations; that happens
in the warm-up.  The result JSON also carries two (b, h) slices of the
reference's O so that bench.py can compare them with this build's output.  This
process never imports this repository's package (both are called
``co_alibi_attn``); it runs as a subprocess of bench.py.
"""
import argparse
import json
import math
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")

CONFIGS = {
    # name: B, Hq, Hkv, S, D, dtype name, causal, input std, fwd_only (as bench.py's CONFIGS)
    "cfg2": (8, 16, 16, 4096, 128, "float16", True, 1.0, False),
    "cfg3": (4, 32, 8, 8192, 128, "bfloat16", True, 1.0, False),
    "cfg4": (16, 12, 12, 2048, 64, "float16", False, 0.5, True),
}


def unit_inputs(torch, cfg, b, g, seed):
    """One (batch element, kv head) unit's inputs; identical to bench.py's
    unit_inputs (same generator, seed and draw order)."""
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    G = Hq // Hkv
    gen = torch.Generator().manual_seed(seed + b * Hkv + g)
    q = (torch.randn(G, S, D, generator=gen) * std).to(dtype)
    k = (torch.randn(1, S, D, generator=gen) * std).to(dtype)
    v = (torch.randn(1, S, D, generator=gen) * std).to(dtype)
    do = torch.randn(G, S, D, generator=gen).to(dtype)
    return q, k, v, do


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seed", type=int, default=1000)
    ap.add_argument("--slices", default="0,0;-1,-1", help="(b, h) pairs of O to return, ';'-separated")
    ap.add_argument("--out", required=True)
    a = ap.parse_args()

    if not os.path.isdir(os.path.join(REF, "co_alibi_attn")):
        raise SystemExit("baseline/_ref/co_alibi_attn is missing: run baseline/install_ref.py first")
    sys.path.insert(0, REF)
    import torch
    import triton
    from co_alibi_attn import co_alibi_attention  # the reference's package
    import co_alibi_attn as ref_pkg
    assert os.path.abspath(ref_pkg.__file__).startswith(REF), ref_pkg.__file__

    B, Hq, Hkv, S, D, dtname, causal, std, fwd_only = CONFIGS[a.config]
    if a.batch:
        B = a.batch
    dtype = getattr(torch, dtname)
    cfg = (B, Hq, Hkv, S, D, dtype, causal, std, fwd_only)
    G = Hq // Hkv
    q = torch.empty(B, Hq, S, D, dtype=dtype)
    k = torch.empty(B, Hkv, S, D, dtype=dtype)
    v = torch.empty(B, Hkv, S, D, dtype=dtype)
    do = torch.empty(B, Hq, S, D, dtype=dtype)
    for b in range(B):
        for g in range(Hkv):
            uq, uk, uv, udo = unit_inputs(torch, cfg, b, g, a.seed)
            q[b, g * G:(g + 1) * G], k[b, g], v[b, g], do[b, g * G:(g + 1) * G] = uq, uk[0], uv[0], udo
    dev = torch.device("cuda", 0)
    q, k, v, do = (t.to(dev) for t in (q, k, v, do))
    scale = 1.0 / math.sqrt(D)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def timed(fn, n):
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    res = {"impl": "reference Triton kernels (baseline/_ref co_alibi_attn.co_alibi_attention, unmodified)",
           "triton": triton.__version__, "config": a.config, "shape": [B, Hq, Hkv, S, D], "dtype": dtname,
           "causal": causal, "steps": a.steps, "warmup": a.warmup}
    t0 = time.time()
    with torch.no_grad():
        for _ in range(a.warmup):
            o = co_alibi_attention(q, k, v, causal=causal, sm_scale=scale)
        torch.cuda.synchronize()
        res["first_calls_s"] = round(time.time() - t0, 1)
        res["fwd_ms"] = timed(lambda: co_alibi_attention(q, k, v, causal=causal, sm_scale=scale), a.steps)
    sl = []
    for pair in a.slices.split(";"):
        b, h = (int(x) for x in pair.split(","))
        b, h = b % B, h % Hq
        sl.append({"b": b, "h": h, "o": o[b, h].float().cpu().tolist()})
    del o
    if not fwd_only:
        qb, kb, vb = (t.clone().requires_grad_(True) for t in (q, k, v))

        def zero():
            for t in (qb, kb, vb):
                if t.grad is not None:
                    t.grad.zero_()

        out = co_alibi_attention(qb, kb, vb, causal=causal, sm_scale=scale)
        for _ in range(a.warmup):
            zero()
            out.backward(do, retain_graph=True)

        def bwd():
            zero()
            out.backward(do, retain_graph=True)

        res["bwd_ms"] = timed(bwd, a.steps)
        del out
        qb.grad = kb.grad = vb.grad = None

        def fwd_bwd():
            o2 = co_alibi_attention(qb, kb, vb, causal=causal, sm_scale=scale)
            o2.backward(do)
            qb.grad = kb.grad = vb.grad = None

        for _ in range(a.warmup):
            fwd_bwd()
        res["fwd_bwd_ms"] = timed(fwd_bwd, a.steps)
    res["peak_mem_gb"] = round(torch.cuda.max_memory_allocated(dev) / 2**30, 2)
    res["slices"] = sl
    with open(a.out, "w") as f:
        json.dump(res, f)


if __name__ == "__main__":
    main()
