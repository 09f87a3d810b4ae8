"""Benchmark of the Co-ALiBi hot path (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg2|cfg3|cfg4|cfg5|decode|cp] [--scaling weak|strong]

One step = co_alibi_attention(q, k, v, causal) forward and backward over one
batch of the named configuration (default cfg2: B=8, H=16, S=4096, D=128, fp16,
causal -- the reference README's bench shape at the baseline batch).  Inputs are
seeded synthetic N(0, std) tensors drawn on the CPU, one generator per (batch
element, kv head) unit, and copied to the GPU; all of them (512 MiB at cfg2)
exceed the 126 MB L2, so no flush is needed between steps.  N>1 runs one process
per GPU under torchrun; every rank runs its own (b, h) units with no collective
on the data path ("strong", the default: the config's fixed batch of B*Hkv units
split into one contiguous block per rank; "weak": every rank holds a full batch).
Time is taken with CUDA events on the launching stream, between a barrier and a
synchronize, and the maximum over ranks is reported.  After timing, NCCL gathers
every rank's outputs for verification (against a single-GPU run of the whole
batch on rank 0 and against the CPU oracle on sampled slices).  At N=1 the
reference's own Triton kernels (baseline/triton_ref.py) are timed on the same
inputs in a subprocess.

``--config cfg5`` instead times one data-parallel training step of the small
Co-ALiBi GPT (co_alibi_gpt: 12 layers, d_model 768, 12 heads of D=64, seq 1024,
batch 32 per GPU, bf16, DDP over NCCL, AdamW) and reports tokens per second.
``--config decode`` times one new query row against a 32,768-key cache;
``--config cp`` one 65,536-token causal sequence split over the N GPUs
(context parallelism, ring over NCCL).

Prints ONE JSON line (rank 0).  ``--impl reference`` times the reference
algorithm's CPU path (the oracle restatement of model.py, on all host cores)
on a bounded sample of the same workload and prints the same metric.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "co-alibi_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

CONFIGS = {
    # name: B, Hq, Hkv, S, D, dtype, causal, input std, fwd_only
    "cfg2": (8, 16, 16, 4096, 128, torch.float16, True, 1.0, False),
    "cfg3": (4, 32, 8, 8192, 128, torch.bfloat16, True, 1.0, False),
    "cfg4": (16, 12, 12, 2048, 64, torch.float16, False, 0.5, True),
}

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of each
# kernel at cfg2: one ncu capture at B=2 (profiles/<kernel>_kernel_cfg2_b2_ncu_full.txt)
# scaled by 4 to the B=8 launch (traffic grows with the number of (b, h) units).
# Pass A and pass B are the stored path's (pass A writes the P / dS tiles pass B reads).
NCU_TRAFFIC_CFG2 = {"fwd": 4 * 117.26e6, "bwd_a": 4 * 1229.95e6, "bwd_b": 4 * 1244.0e6, "bwd_delta": None}


def visible(S, causal):
    return S * (S + 1) // 2 if causal else S * S


def unit_inputs(cfg, b, g, seed=1000):
    """Inputs of one (batch element b, kv head g) unit -- K and V of the kv head, Q
    and dO of its G query heads -- from a CPU generator seeded by the unit's index,
    so every rank draws exactly its own units of one global batch (and
    baseline/triton_ref.py the same batch)."""
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    G = Hq // Hkv
    gen = torch.Generator().manual_seed(seed + b * Hkv + g)
    q = (torch.randn(G, S, D, generator=gen) * std).to(dtype)
    k = (torch.randn(1, S, D, generator=gen) * std).to(dtype)
    v = (torch.randn(1, S, D, generator=gen) * std).to(dtype)
    do = torch.randn(G, S, D, generator=gen).to(dtype)
    return q, k, v, do


def shard_inputs(cfg, b0, b1, g0, g1, pin=False):
    """(q, k, v, do) host tensors of units b0 <= b < b1, g0 <= g < g1."""
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    G = Hq // Hkv
    mk = lambda h: torch.empty(b1 - b0, h, S, D, dtype=dtype, pin_memory=pin)  # noqa: E731
    q, k, v, do = mk((g1 - g0) * G), mk(g1 - g0), mk(g1 - g0), mk((g1 - g0) * G)
    for b in range(b0, b1):
        for g in range(g0, g1):
            uq, uk, uv, udo = unit_inputs(cfg, b, g)
            i, j = b - b0, g - g0
            q[i, j * G:(j + 1) * G], k[i, j], v[i, j], do[i, j * G:(j + 1) * G] = uq, uk[0], uv[0], udo
    return q, k, v, do


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), d.get("hbm_gbs"), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.base = 0

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # return once nvidia-smi is sampling, and count only the samples taken
            # after this point (inside the timed region)
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.base = len(self.lines)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        lines = self.lines[self.base:]
        if not lines:
            # a timed region shorter than the sampling period: one reading right after it
            try:
                r = subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                    "-i", str(self.idx)], capture_output=True, text=True, timeout=10)
                lines = [ln.strip() for ln in r.stdout.splitlines()]
            except Exception:
                lines = []
        mhz, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(mhz)}


def physical_gpu_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p.strip() for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].isdigit():
            return int(parts[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# CPU side: the oracle restatement of the reference's model.py
# ---------------------------------------------------------------------------
def cpu_sample_tflops(cfg, rows, reps, threads=None):
    """Time fwd+bwd of the oracle (model.py maths, fp32, all host threads) on the
    last `rows` query rows of one (b, h) slice of the config.  Returns (TFLOP/s,
    seconds per sample, threads, description)."""
    from oracle import coalibi_oracle as orc
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    if threads:
        torch.set_num_threads(threads)
    nthreads = torch.get_num_threads()
    g = torch.Generator().manual_seed(1)
    q = (torch.randn(1, 1, rows, D, generator=g) * std).to(dtype)
    k = (torch.randn(1, 1, S, D, generator=g) * std).to(dtype)
    v = (torch.randn(1, 1, S, D, generator=g) * std).to(dtype)
    do = torch.randn(1, 1, rows, D, generator=g).to(dtype)
    sl = orc.api_slopes(Hq, 8.0, dtype)[:1]
    off = S - rows
    f, b = orc.algorithmic_flops(1, 1, rows, S, D, causal, q_offset=off)
    flops = f if fwd_only else f + b
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        if fwd_only:
            orc.forward(q, k, v, sl, causal, None, torch.float32, q_offset=off)
        else:
            orc.forward_backward(q, k, v, do, sl, causal, None, torch.float32, q_offset=off)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    desc = (f"oracle (model.py maths) fp32 {'fwd' if fwd_only else 'fwd+bwd'} on one (b,h) slice, "
            f"query rows {off}..{S - 1} of S={S}, D={D}, median of {reps}")
    return flops / t / 1e12, t, nthreads, desc


def flash_side_by_side(cfg, dev, steps, warmup):
    """FlashAttention-2 (flash_attn_func, the library's kernels) on the config's
    shape and inputs, as the reference's benchmark_flops.py:94-136 does optionally:
    layout [B, S, H, D], same scale and mask, CUDA events around `steps` forward
    calls and `steps` forward + backward steps.  A comparator only: it computes
    softmax attention without the Co-ALiBi bias.  Returns a dict, or the reason it
    could not run."""
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    try:
        from flash_attn import flash_attn_func
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flash_attn import failed: {type(e).__name__}: {e}"[:200]}
    import flash_attn
    g = torch.Generator().manual_seed(7)
    q = (torch.randn(B, S, Hq, D, generator=g) * std).to(dtype).to(dev).requires_grad_(True)
    k = (torch.randn(B, S, Hkv, D, generator=g) * std).to(dtype).to(dev).requires_grad_(True)
    v = (torch.randn(B, S, Hkv, D, generator=g) * std).to(dtype).to(dev).requires_grad_(True)
    do = torch.randn(B, S, Hq, D, generator=g).to(dtype).to(dev)
    scale = 1.0 / math.sqrt(D)

    def fwd():
        with torch.no_grad():
            flash_attn_func(q, k, v, softmax_scale=scale, causal=causal)

    def fwd_bwd():
        o = flash_attn_func(q, k, v, softmax_scale=scale, causal=causal)
        o.backward(do)
        q.grad = k.grad = v.grad = None

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    try:
        fwd_ms = timed(fwd)
        step_ms = None if fwd_only else timed(fwd_bwd)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flash_attn on this GPU: {type(e).__name__}: {e}"[:200]}
    E = visible(S, causal) * B * Hq
    out = {"impl": f"flash_attn {flash_attn.__version__} flash_attn_func (FlashAttention-2, softmax without the "
                   f"Co-ALiBi bias)", "fwd_ms": round(fwd_ms, 4), "fwd_tflops": round(4.0 * D * E / fwd_ms / 1e9, 2)}
    if step_ms is not None:
        out.update({"fwd_bwd_ms": round(step_ms, 4), "fwd_bwd_tflops": round(14.0 * D * E / step_ms / 1e9, 2)})
    del q, k, v, do
    torch.cuda.empty_cache()
    return out


def pcie_copy_floor_ms(ins_h, outs_h, dev, reps=3):
    """Time of the e2e step's transfers alone: every input copied host -> device on
    one stream while every output is copied device -> host on another (both PCIe
    directions at once), no kernels; the floor under the e2e number."""
    ins_d = [torch.empty_like(h, device=dev) for h in ins_h]
    outs_d = [torch.empty_like(h, device=dev) for h in outs_h]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    best = float("inf")
    for _ in range(reps + 1):
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            for d, h in zip(ins_d, ins_h):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            for h, d in zip(outs_h, outs_d):
                h.copy_(d, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        e1.record(cur)
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1))
    del ins_d, outs_d
    return best


def verify_shards(cfg, shard, world, rank, dev, qd, kd, vd, dod, attn, oracle_slices=2):
    """Verification of the (b, h)-sharded run, outside the timed region: every rank
    runs its shard once more, NCCL all-gathers the shards' o / dq / dk / dv (the only
    use of a collective on data), and rank 0 compares the gathered batch with a
    single-GPU run of the whole batch (at N > 1) and with the CPU oracle on
    `oracle_slices` (b, h) slices of the first and last ranks' shards.  Returns the
    summary on rank 0, None elsewhere."""
    import torch.distributed as dist
    import co_alibi_attn
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    G = Hq // Hkv
    qg = qd.detach().clone().requires_grad_(not fwd_only)
    kg = kd.detach().clone().requires_grad_(not fwd_only)
    vg = vd.detach().clone().requires_grad_(not fwd_only)
    if fwd_only:
        with torch.no_grad():
            outs = [attn(qg, kg, vg)]
    else:
        o = attn(qg, kg, vg)
        o.backward(dod)
        outs = [o.detach(), qg.grad, kg.grad, vg.grad]
    torch.cuda.synchronize()
    names = ["o", "dq", "dk", "dv"][:len(outs)]
    # gather: every rank's shard of each output, in rank order (equal sizes by construction)
    gathered = []
    for t in outs:
        t = t.contiguous()
        if world > 1:
            buf = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=dev)
            dist.all_gather_into_tensor(buf, t)
        else:
            buf = t.unsqueeze(0)
        gathered.append(buf)
    torch.cuda.synchronize()
    if rank != 0:
        return None
    from co_alibi_attn.sharding import shard_plan
    plans = [shard_plan(B, Hq, Hkv, world, r) if world > 1 else shard for r in range(world)]

    def assemble(i):
        """The whole batch's output i from the gathered shards (host)."""
        heads = Hq if names[i] in ("o", "dq") else Hkv
        per = G if heads == Hq else 1
        full = torch.empty(B, heads, S, D, dtype=dtype)
        for r, sh in enumerate(plans):
            full[sh.b0:sh.b1, sh.g0 * per:sh.g1 * per] = gathered[i][r].cpu()
        return full

    full = [assemble(i) for i in range(len(names))]
    out = {"collective": f"NCCL all_gather_into_tensor of each rank's {'/'.join(names)} shard" if world > 1
           else "none (one rank)", "ranks": world}
    if world > 1:
        # rank 0 alone runs the whole batch through the public API and compares
        q1, k1, v1, do1 = (t.to(dev) for t in shard_inputs(cfg, 0, B, 0, Hkv))
        q1.requires_grad_(not fwd_only), k1.requires_grad_(not fwd_only), v1.requires_grad_(not fwd_only)
        if fwd_only:
            with torch.no_grad():
                ref = [co_alibi_attn.co_alibi_attention(q1, k1, v1, causal=causal)]
        else:
            o1 = co_alibi_attn.co_alibi_attention(q1, k1, v1, causal=causal)
            o1.backward(do1)
            ref = [o1.detach(), q1.grad, k1.grad, v1.grad]
        torch.cuda.synchronize()
        cmp = {}
        for n, a, r in zip(names, full, ref):
            r = r.cpu()
            cmp[n] = {"bitwise_equal": bool(torch.equal(a, r)),
                      "max_abs_diff": float((a.float() - r.float()).abs().max())}
        out["vs_single_gpu_whole_batch"] = cmp
        del q1, k1, v1, do1, ref
    # the CPU oracle on sampled slices (first unit of rank 0, last unit of the last rank)
    sys.path.insert(0, ROOT)
    from oracle import coalibi_oracle as orc
    torch.set_num_threads(os.cpu_count() or 1)
    sl = orc.api_slopes(Hq, 8.0, dtype)
    picks = [(0, 0), (B - 1, Hq - 1)][:oracle_slices]
    res = []
    for (b, h) in picks:
        g = h // G
        uq, uk, uv, udo = unit_inputs(cfg, b, g)
        qs, ks, vs, dos = uq[h - g * G][None, None], uk[None], uv[None], udo[h - g * G][None, None]
        r = {"b": b, "h": h}
        if fwd_only:
            o_r, _, _ = orc.forward(qs, ks, vs, sl[h:h + 1], causal, None, torch.float32)
        else:
            o_r, _, _, dq_r, dk_r, dv_r = orc.forward_backward(qs, ks, vs, dos, sl[h:h + 1], causal, None,
                                                               torch.float32)
        r["o_max_abs"] = float((full[0][b, h].double() - o_r[0, 0].double()).abs().max())
        if not fwd_only:
            rel = lambda x, y: float((x.double() - y.double()).norm() / y.double().norm())  # noqa: E731
            r["dq_rel"] = rel(full[1][b, h], dq_r[0, 0])
            if G == 1:  # dk / dv of one query head equal the kv head's only when no group sum is needed
                r["dk_rel"] = rel(full[2][b, g], dk_r[0, 0])
                r["dv_rel"] = rel(full[3][b, g], dv_r[0, 0])
        res.append(r)
    o_tol = 2e-3 if dtype == torch.float16 else 2e-2
    ok = all(r["o_max_abs"] <= o_tol and all(r.get(n, 0.0) <= 1e-2 for n in ("dq_rel", "dk_rel", "dv_rel"))
             for r in res)
    out["vs_oracle"] = {"slices": res, "o_tol": o_tol, "grad_rel_tol": 1e-2, "pass": ok,
                        "oracle": "fp32 CPU restatement of model.py (oracle/), one (b, h) slice each"}
    out["pass"] = ok and all(c["bitwise_equal"] or c["max_abs_diff"] == 0.0
                             for c in out.get("vs_single_gpu_whole_batch", {}).values())
    return out


def reference_triton_side_by_side(args, cfg, o_ours, ms_ours, fwd_ms_ours, timeout_s=900):
    """The reference's own Triton kernels on the same inputs and GPU, run by
    baseline/triton_ref.py in a subprocess (both packages are named co_alibi_attn).
    Returns its timings, this build's speed-up over them, and the largest
    difference between its O and this build's on two (b, h) slices."""
    import tempfile
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    script = os.path.join(ROOT, "baseline", "triton_ref.py")
    if not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "co_alibi_attn")):
        return {"unavailable": "baseline/_ref holds no reference package (python baseline/install_ref.py "
                               "<reference checkout> installs it)"}
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "ref.json")
        cmd = [sys.executable, script, "--config", args.config, "--steps", str(max(3, min(args.steps, 10))),
               "--warmup", "3", "--out", out]
        if args.batch:
            cmd += ["--batch", str(args.batch)]
        env = dict(os.environ)
        env.pop("COALIBI_VERBOSE", None)
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s, env=env)
        except subprocess.TimeoutExpired:
            return {"unavailable": f"baseline/triton_ref.py did not finish within {timeout_s} s"}
        if r.returncode != 0 or not os.path.exists(out):
            tail = (r.stderr.strip().splitlines() or ["(no output)"])[-1]
            return {"unavailable": f"baseline/triton_ref.py exited {r.returncode}: {tail}"[:300]}
        with open(out) as f:
            ref = json.load(f)
    E = visible(S, causal) * B * Hq
    res = {k: ref[k] for k in ("impl", "triton", "first_calls_s", "peak_mem_gb") if k in ref}
    res["fwd_ms"] = round(ref["fwd_ms"], 4)
    res["fwd_tflops"] = round(4.0 * D * E / (ref["fwd_ms"] * 1e-3) / 1e12, 2)
    if fwd_ms_ours:
        res["fwd_speedup_of_this_build"] = round(ref["fwd_ms"] / fwd_ms_ours, 2)
    if "bwd_ms" in ref:
        res["bwd_ms"] = round(ref["bwd_ms"], 4)
        res["bwd_tflops"] = round(10.0 * D * E / (ref["bwd_ms"] * 1e-3) / 1e12, 2)
        res["bwd_note"] = "backward(retain_graph=True) replayed on one graph, gradients zeroed each time " \
                          "(the reference benchmark's convention, co_alibi_attn/benchmark_flops.py:66-92)"
    if "fwd_bwd_ms" in ref:
        res["fwd_bwd_ms"] = round(ref["fwd_bwd_ms"], 4)
        res["fwd_bwd_tflops"] = round(14.0 * D * E / (ref["fwd_bwd_ms"] * 1e-3) / 1e12, 2)
        res["fwd_bwd_speedup_of_this_build"] = round(ref["fwd_bwd_ms"] / ms_ours, 2)
    diffs = []
    for s_ in ref.get("slices", []):
        o_ref = torch.tensor(s_["o"])
        diffs.append({"b": s_["b"], "h": s_["h"],
                      "o_max_abs_diff_vs_this_build": float((o_ours[s_["b"], s_["h"]].float() - o_ref).abs().max())})
    res["o_compare"] = diffs
    res["tflops_note"] = "algorithmic causal FLOPs (4 D forward, 10 D backward per visible score), as for this build"
    return res


def run_reference_arm(args, cfg, rank):
    if rank != 0:
        return
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    # size each step so that warmup + steps fit in about two minutes
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = S
    _, t, _, _ = cpu_sample_tflops(cfg, min(S, 512), 1)
    per_row = t / min(S, 512)
    while rows > 64 and rows * per_row * 1.5 > budget:
        rows //= 2
    from oracle import coalibi_oracle as orc
    tfl, tsec, nthreads, desc = cpu_sample_tflops(cfg, rows, args.warmup + args.steps)
    ms = tsec * 1e3
    line = {
        "impl": "reference", "metric": metric_name(args.config), "value": round(tfl, 6), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_dict(args, cfg),
        "cpu_baseline": {"value": round(tfl, 6), "unit": "TFLOP/s", "cores": nthreads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(tfl, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference arm: the reference's own CPU path (model.py maths) restated in oracle/, "
                "timed on the host cores; the reference's Triton GPU kernels are timed on the same GPU by "
                "the default arm (its reference_triton key, from baseline/_ref when installed)",
    }
    print(json.dumps(line), flush=True)


def run_gpt(args, world, rank, local_rank, dev):
    """cfg5: one data-parallel training step of the small Co-ALiBi GPT per step
    (forward, backward with the NCCL gradient all-reduce of DDP, AdamW update);
    value = tokens per second over all ranks."""
    import torch.distributed as dist
    import co_alibi_attn
    import co_alibi_attn.co_alibi_attn as impl
    from co_alibi_gpt import GPTConfig, build, make_tokens, train_step
    cfg = GPTConfig()
    batch = args.batch or 32

    def barrier():
        if world > 1:
            dist.barrier()

    model, opt = build(cfg, dev, seed=0, ddp=world > 1)
    core = model.module if world > 1 else model
    tok_h = make_tokens(cfg, batch, seed=1000 + rank).pin_memory()
    tok = tok_h.to(dev)
    for _ in range(args.warmup):
        train_step(model, opt, tok)
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0, "kernel-side error during warmup"

    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        train_step(model, opt, tok)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = t.item()
    tokens_rank = batch * cfg.seq_len
    value = world * tokens_rank / (ms_max * 1e-3)
    flops_rank = core.flops_per_token() * tokens_rank
    burst, sustained, hbm, peak_src = load_peaks()
    achieved = flops_rank / (ms_max * 1e-3) / 1e12

    # attention kernels inside a step (CUDA events around each launch, separate short pass)
    impl.kernel_events = {}
    for _ in range(3):
        train_step(model, opt, tok)
    torch.cuda.synchronize()
    attn_ms = sum(a.elapsed_time(b) for v in impl.kernel_events.values() for a, b in v) / 3
    impl.kernel_events = None
    attn_flops = cfg.n_layer * 14 * cfg.d_model * (cfg.seq_len + 1) / 2 * tokens_rank

    # e2e: token ids from pinned host memory every step, the loss read back every step
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    tok_d = torch.empty_like(tok)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    n_e2e = max(1, args.e2e_steps)
    for _ in range(n_e2e):
        tok_d.copy_(tok_h, non_blocking=True)
        loss = train_step(model, opt, tok_d)
        loss_h.copy_(loss.float(), non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    t = torch.tensor([f0.elapsed_time(f1) / n_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = t.item()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = gpt_cpu_sample(cfg)
    if rank == 0:
        line = {
            "metric": metric_name("cfg5"), "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (token ids uniform over the vocabulary, weights N(0, 0.02))",
            "config": {"workload": f"cfg5: Co-ALiBi GPT training step, {cfg.n_layer} layers, d_model {cfg.d_model}, "
                                   f"{cfg.n_head} heads (D=64), MLP 4x GELU, vocab {cfg.vocab}, seq {cfg.seq_len}, "
                                   f"batch {batch} per GPU, bf16 weights, AdamW",
                       "global_batch": world * batch, "seq_len": cfg.seq_len,
                       "parallelism": f"data-parallel x{world} (DDP, NCCL all-reduce of bf16 gradients)",
                       "l2": "weights, activations and optimizer state exceed the 126 MB L2"},
            "model_tflops_per_gpu": round(achieved, 2),
            "attention": {"ms_per_step": round(attn_ms, 3), "share": round(attn_ms / ms_max, 4),
                          "tflops": round(attn_flops / (attn_ms * 1e-3) / 1e12, 2) if attn_ms > 0 else None},
            "roofline": {"bound": "tensor", "kernel": "whole training step (GEMMs + Co-ALiBi attention)",
                         "achieved": round(achieved, 2), "peak": sustained, "unit": "TFLOP/s",
                         "frac": round(achieved / sustained, 4),
                         "peak_source": f"{peak_src} bf16_tflops_sustained", "traffic": None,
                         "note": "6 x matmul parameters per token + causal attention GEMMs, per GPU"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * tokens_rank / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": tok_h.numel() * tok_h.element_size(), "d2h_bytes_per_step": 4},
            "gpu_launches": 4 * cfg.n_layer * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)


def run_decode(args, world, rank, local_rank, dev):
    """decode: one new query row per (batch, head) against a 32,768-key cache
    (B=8, Hq=32, Hkv=8, D=128, bf16, no mask) through co_alibi_attention, which
    takes the split-over-keys decode kernels for Sq <= 16.  value = query rows
    (generated tokens x heads / heads = tokens) per second over all ranks."""
    import torch.distributed as dist
    import co_alibi_attn
    from co_alibi_attn import co_alibi_attention
    import co_alibi_attn.co_alibi_attn as impl
    B, Hq, Hkv, Sq, Skv, D, dt = (args.batch or 8), 32, 8, 1, 32768, 128, torch.bfloat16

    def barrier():
        if world > 1:
            dist.barrier()

    g = torch.Generator().manual_seed(2000 + rank)
    q_h = torch.randn(B, Hq, Sq, D, generator=g).to(dt).pin_memory()
    k = torch.randn(B, Hkv, Skv, D, generator=g).to(dt).to(dev)
    v = torch.randn(B, Hkv, Skv, D, generator=g).to(dt).to(dev)
    q = q_h.to(dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            co_alibi_attention(q, k, v, causal=False)
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0, "kernel-side error during warmup"
    # K, V (2 x 1 GiB) exceed the L2: every call reads them from HBM
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        e0.record()
        for _ in range(args.steps):
            co_alibi_attention(q, k, v, causal=False)
        e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = t.item()
    bytes_call = (k.numel() + v.numel() + 2 * q.numel()) * 2
    burst, sustained, hbm, peak_src = load_peaks()
    gbs = bytes_call / (ms_max * 1e-3) / 1e9
    # decode partial kernel alone (CUDA events around the launch pair)
    impl.kernel_events = {}
    with torch.no_grad():
        for _ in range(5):
            co_alibi_attention(q, k, v, causal=False)
    torch.cuda.synchronize()
    kms = sum(a.elapsed_time(b) for a, b in impl.kernel_events.get("fwd", [])) / 5
    impl.kernel_events = None
    # e2e: the new query rows from pinned host memory, the output read back, every call
    o_h = torch.empty_like(q_h).pin_memory()
    qd = torch.empty_like(q)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(1, args.e2e_steps)
    with torch.no_grad():
        f0.record()
        for _ in range(n_e2e):
            qd.copy_(q_h, non_blocking=True)
            o = co_alibi_attention(qd, k, v, causal=False)
            o_h.copy_(o, non_blocking=True)
        f1.record()
    torch.cuda.synchronize()
    t = torch.tensor([f0.elapsed_time(f1) / n_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = t.item()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import coalibi_oracle as orc
        torch.set_num_threads(os.cpu_count() or 1)
        sl = orc.api_slopes(Hq, 8.0, torch.float32)[:1]
        qs, ks, vs = q_h[:1, :1].float(), k[:1, :1].float().cpu(), v[:1, :1].float().cpu()
        orc.forward(qs, ks, vs, sl, False, None, torch.float32)
        t0 = time.perf_counter()
        for _ in range(5):
            orc.forward(qs, ks, vs, sl, False, None, torch.float32)
        sec = (time.perf_counter() - t0) / 5
        cpu = {"value": round(1.0 / sec, 1), "unit": "query rows/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"oracle (model.py maths) fp32, one query row of one head against {Skv} keys, mean of 5",
               "seconds_per_sample": round(sec, 6)}
    if rank == 0:
        rows = B * Hq * Sq
        line = {
            "metric": metric_name("decode"), "value": round(world * rows / (ms_max * 1e-3), 1), "unit": "query rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"decode: co_alibi_attention fwd, B={B} Hq={Hq} Hkv={Hkv} Sq={Sq} Skv={Skv} D={D} "
                                   "bf16, no mask (one new token per sequence against the key/value cache)",
                       "global_batch": world * B, "seq_len": Skv, "parallelism": f"independent replicas x{world}",
                       "l2": "K and V (2 GiB) exceed the 126 MB L2; no flush needed"},
            "kv_read_gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "kernel": "decode (partial + combine)", "achieved": round(gbs, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4), "peak_source": f"{peak_src} hbm_gbs",
                         "traffic": None, "kernel_ms": round(kms, 4),
                         "note": "K + V + Q + O bytes per call / CUDA-event time of the call"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * rows / (e2e_ms * 1e-3), 1), "unit": "query rows/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": q_h.numel() * 2, "d2h_bytes_per_step": o_h.numel() * 2},
            "gpu_launches": 2 * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)


CP_SHAPE = (1, 32, 8, 65536, 128)   # B, Hq, Hkv, S, D of the context-parallel line


def run_cp(args, world, rank, local_rank, dev):
    """cp: one long causal sequence (B=1, Hq=32, Hkv=8, S=65,536, D=128, bf16)
    forward + backward through context_parallel.ring_attention with the zig-zag
    layout: the sequence in 2N chunks, rank r holding chunks r and 2N-1-r, key /
    value chunks (and dk / dv accumulators) passed around the NCCL ring.  Total
    work is fixed ("strong"); value = the whole sequence's algorithmic FLOPs per
    second."""
    import torch.distributed as dist
    import co_alibi_attn
    import co_alibi_attn.co_alibi_attn as impl
    from co_alibi_attn.context_parallel import chunk_layout, ring_attention
    B, Hq, Hkv, S, D = CP_SHAPE
    if args.seq_len:
        S = args.seq_len
        if S % (2 * world * 128):
            raise SystemExit(f"--seq-len must be a multiple of {2 * world * 128} at N={world}")
    dt = torch.bfloat16
    own = chunk_layout("zigzag", world, rank)
    L = S // (2 * world)

    def barrier():
        if world > 1:
            dist.barrier()

    def chunk(i):
        g = torch.Generator().manual_seed(3000 + i)
        return (torch.randn(B, Hq, L, D, generator=g).to(dt), torch.randn(B, Hkv, L, D, generator=g).to(dt),
                torch.randn(B, Hkv, L, D, generator=g).to(dt), torch.randn(B, Hq, L, D, generator=g).to(dt))

    parts = [chunk(i) for i in own]
    hosts = [torch.cat([p[j] for p in parts], dim=2).pin_memory() for j in range(4)]
    q, k, v, do = (h.to(dev) for h in hosts)
    for t in (q, k, v):
        t.requires_grad_(True)

    def step():
        o = ring_attention(q, k, v, causal=True, layout="zigzag")
        o.backward(do)
        q.grad = k.grad = v.grad = None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0, "kernel-side error during warmup"
    impl.kernel_events = {}
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    rec = impl.kernel_events
    impl.kernel_events = None
    status = co_alibi_attn.device_status(reset=True)
    ms = e0.elapsed_time(e1) / args.steps
    kern = {name: sum(a.elapsed_time(b) for a, b in pairs) / args.steps for name, pairs in rec.items()}
    launches = {name: len(pairs) // args.steps for name, pairs in rec.items()}
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = t.item()
    E_all = visible(S, True) * B * Hq
    flops_step = 14.0 * D * E_all
    value = flops_step / (ms_max * 1e-3) / 1e12
    # this rank's visible scores: pairs (i, j <= i) of its chunks against all chunks
    E_rank = sum((i * L * L + L * (L + 1) // 2) for i in own) * B * Hq
    kern_ms = kern.get("fwd", 0.0) + kern.get("bwd_carry", 0.0)
    ach = 14.0 * D * E_rank / (kern_ms * 1e-3) / 1e12
    # e2e: this rank's chunks from pinned host memory, o / dq / dk / dv back, every step
    outs = [torch.empty_like(hosts[0]).pin_memory(), torch.empty_like(hosts[0]).pin_memory(),
            torch.empty_like(hosts[1]).pin_memory(), torch.empty_like(hosts[2]).pin_memory()]
    qd, kd, vd, dod = (torch.empty_like(x) for x in (q, k, v, do))

    phase_events = []  # per e2e step: events before the copies in, after them, after the ring, after the copies out

    def e2e_step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        for dst, src in zip((qd, kd, vd, dod), hosts):
            dst.copy_(src, non_blocking=True)
        ev[1].record()
        qi, ki, vi = (x.detach().requires_grad_(True) for x in (qd, kd, vd))
        o = ring_attention(qi, ki, vi, causal=True, layout="zigzag")
        o.backward(dod)
        ev[2].record()
        for dst, src in zip(outs, (o, qi.grad, ki.grad, vi.grad)):
            dst.copy_(src, non_blocking=True)
        ev[3].record()
        phase_events.append(ev)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    phase_events.clear()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(1, args.e2e_steps)
    f0.record()
    for _ in range(n_e2e):
        e2e_step()
    f1.record()
    torch.cuda.synchronize()
    # where an e2e step's time goes on this rank (mean over the steps), then the max over ranks
    phases = torch.tensor([sum(e[i].elapsed_time(e[i + 1]) for e in phase_events) / n_e2e for i in range(3)],
                          device=dev)
    t = torch.tensor([f0.elapsed_time(f1) / n_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(phases, op=dist.ReduceOp.MAX)
    e2e_ms = t.item()
    e2e_phases = {"h2d_ms": round(phases[0].item(), 3), "ring_fwd_bwd_ms": round(phases[1].item(), 3),
                  "d2h_ms": round(phases[2].item(), 3),
                  "note": "CUDA events on each rank's stream around its copies in, ring forward + backward and "
                          "copies out, mean over the e2e steps, max over ranks"}
    burst, sustained, hbm, peak_src = load_peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tfl, tsec, nth, desc = cpu_sample_tflops((B, Hq, Hkv, S, D, dt, True, 1.0, False), 256, 3)
        cpu = {"value": round(tfl, 6), "unit": "TFLOP/s", "cores": nth, "kind": "port", "sample": desc,
               "seconds_per_sample": round(tsec, 3)}
    if rank == 0:
        line = {
            "metric": metric_name("cp") if S == CP_SHAPE[3] else metric_name("cp").replace("S65536", f"S{S}"),
            "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cp: ring_attention fwd+bwd (context parallel, zig-zag chunks), B={B} Hq={Hq} "
                                   f"Hkv={Hkv} S={S} D={D} bf16 causal", "global_batch": B, "seq_len": S,
                       "parallelism": f"sequence x{world} ({2 * world} zig-zag chunks, NCCL ring)",
                       "l2": f"q, do ({q.numel() * 2 >> 20} MiB each on this rank) "
                             + ("exceed the 126 MB L2; no flush needed" if q.numel() * 2 > 126e6 else
                                "fit the 126 MB L2: a capture size, not a bench line")},
            "roofline": {"bound": "tensor", "kernel": "fwd + bwd_carry pair kernels (rank 0)", "achieved": round(ach, 2),
                         "peak": sustained, "unit": "TFLOP/s", "frac": round(ach / sustained, 4),
                         "peak_source": f"{peak_src} bf16_tflops_sustained", "traffic": None,
                         "kernel_ms": round(kern_ms, 3), "merge_and_ring_ms": round(ms - kern_ms, 3),
                         "note": "rank 0's algorithmic FLOPs (14 D per visible score) / the summed CUDA-event time "
                                 "of its pair kernels; the rest of the step is the merge arithmetic, the carries and "
                                 "the ring transfers not hidden behind the kernels"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(flops_step / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": sum(h.numel() * 2 for h in hosts),
                    "d2h_bytes_per_step": sum(x.numel() * 2 for x in outs), "phases": e2e_phases},
            "gpu_launches": launches.get("fwd", 0) + 3 * launches.get("bwd_carry", 0),
            "clocks": clocks, "device_status": status,
        }
        print(json.dumps(line), flush=True)


def gpt_cpu_sample(cfg):
    """The same GPT, float32 on the host cores, the attention from the oracle
    (the reference's own maths restated): one sequence forward + backward."""
    from co_alibi_gpt import build, make_tokens
    from oracle import coalibi_oracle as orc
    torch.set_num_threads(os.cpu_count() or 1)

    def attn(q, k, v, causal=True, bias_max=8.0):
        sl = orc.api_slopes(q.shape[1], bias_max, q.dtype)
        return orc.forward(q, k, v, sl, causal, None, torch.float32)[0]

    model, _ = build(cfg, "cpu", seed=0, dtype=torch.float32, attn_fn=attn)
    tok = make_tokens(cfg, 1, seed=7)
    model(tok[:, :-1], targets=tok[:, 1:]).backward()
    model.zero_grad(set_to_none=True)
    t0 = time.perf_counter()
    model(tok[:, :-1], targets=tok[:, 1:]).backward()
    sec = time.perf_counter() - t0
    return {"value": round(cfg.seq_len / sec, 1), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"one sequence of {cfg.seq_len} tokens, forward + backward, float32, "
                                      "attention from the oracle (model.py maths)", "seconds_per_sample": round(sec, 3)}


def metric_name(config):
    return {"cfg2": "fwd+bwd TFLOP/s (algorithmic causal), B8 H16 S4096 D128 fp16 causal",
            "cfg3": "fwd+bwd TFLOP/s (algorithmic causal), GQA B4 Hq32 Hkv8 S8192 D128 bf16 causal",
            "cfg4": "fwd TFLOP/s, B16 H12 S2048 D64 fp16 non-causal",
            "cfg5": "Co-ALiBi GPT training step tokens/s (12 layers, d768, 12 heads D64, seq 1024, batch 32 per GPU)",
            "decode": "decode query rows/s, B8 Hq32 Hkv8 Sq1 Skv32768 D128 bf16",
            "cp": "context-parallel fwd+bwd TFLOP/s (algorithmic causal), B1 Hq32 Hkv8 S65536 D128 bf16"}[config]


def config_dict(args, cfg):
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    units_per_rank = B * Hkv if args.scaling == "weak" else B * Hkv // max(1, args.gpus)
    return {"workload": f"{args.config}: co_alibi_attention {'fwd' if fwd_only else 'fwd+bwd'} B={B} Hq={Hq} "
                        f"Hkv={Hkv} S={S} D={D} {str(dtype).split('.')[-1]} "
                        f"{'causal' if causal else 'non-causal'}",
            "global_batch": B * (args.gpus if args.scaling == "weak" else 1), "seq_len": S,
            "heads": Hq, "kv_heads": Hkv, "head_dim": D, "units_per_rank": units_per_rank,
            "parallelism": (f"(b,h)-shards x{args.gpus} ({args.scaling} scaling: "
                            + ("the fixed batch split over the ranks" if args.scaling == "strong"
                               else "a full batch per rank") + "), no data-path collective"),
            "l2": "inputs (4 x B*H*S*D*2 bytes) exceed the 126 MB L2; no flush needed"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS) + ["cfg5", "decode", "cp"])
    ap.add_argument("--scaling", default="strong", choices=["weak", "strong"],
                    help="strong (default): the config's batch split over the ranks; weak: a full batch per rank")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None,
                    help="override the config's batch size (small cases for ncu captures)")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="--config cp only: override the sequence length (small cases for ncu captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-side-by-side", action="store_true",
                    help="skip the FlashAttention-2 and reference-Triton comparisons on the same shape (N=1 only)")
    ap.add_argument("--no-verify", action="store_true",
                    help="skip the post-timing verification gather (small ncu capture cases)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config in ("cfg5", "decode", "cp"):
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                why = {"cfg5": "the reference ships no model code; cfg5 is a caller built here",
                       "decode": "the decode line is an addition of this build; the reference arm is the default config's",
                       "cp": "the reference has no sequence parallelism; the reference arm is the default config's"
                       }[args.config]
                print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
            return
        cfg = None
    else:
        cfg = CONFIGS[args.config]
        if args.batch:
            cfg = (args.batch,) + cfg[1:]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, cfg, rank)
        return

    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        # communicator creation prints a "NCCL version" line on the process's stdout
        # (C-level, not sys.stdout); point fd 1 at stderr meanwhile so stdout carries
        # only the JSON line
        sys.stdout.flush()
        saved_fd = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
            dist.barrier(device_ids=[local_rank])
            torch.cuda.synchronize()
        finally:
            os.dup2(saved_fd, 1)
            os.close(saved_fd)

    if args.config in ("cfg5", "decode", "cp"):
        {"cfg5": run_gpt, "decode": run_decode, "cp": run_cp}[args.config](args, world, rank, local_rank, dev)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    import co_alibi_attn
    from co_alibi_attn import co_alibi_attention
    import co_alibi_attn.co_alibi_attn as impl

    from co_alibi_attn.sharding import shard_plan, sharded_attention, shard_slopes
    B, Hq, Hkv, S, D, dtype, causal, std, fwd_only = cfg
    if args.scaling == "strong" and world > 1:
        # the batch's B*Hkv (b, kv head) units split into one contiguous block per rank
        shard = shard_plan(B, Hq, Hkv, world, rank)
    else:
        shard = shard_plan(B, Hq, Hkv, 1, 0)
    B_r, Hq_r, Hkv_r = shard.b1 - shard.b0, shard.h1 - shard.h0, shard.g1 - shard.g0

    def attn(q_, k_, v_):
        if args.scaling == "strong" and world > 1:
            return sharded_attention(q_, k_, v_, shard, Hq, causal=causal)
        return co_alibi_attention(q_, k_, v_, causal=causal)

    # weak scaling: every rank holds the whole batch (the same units); strong: its block
    q_h, k_h, v_h, do_h = shard_inputs(cfg, shard.b0, shard.b1, shard.g0, shard.g1, pin=True)
    q = q_h.to(dev).requires_grad_(not fwd_only)
    k = k_h.to(dev).requires_grad_(not fwd_only)
    v = v_h.to(dev).requires_grad_(not fwd_only)
    do = do_h.to(dev)

    E = visible(S, causal) * B_r * Hq_r
    flops_fwd = 4.0 * D * E
    flops_step = flops_fwd if fwd_only else 14.0 * D * E
    kernels_per_step = 1 if fwd_only else 4

    def step():
        if fwd_only:
            with torch.no_grad():
                attn(q, k, v)
        else:
            o = attn(q, k, v)
            o.backward(do)
            q.grad = k.grad = v.grad = None

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0, "kernel-side error during warmup"

    # ---------------- timed region: the public API alone, K steps back to back
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # host time to enqueue a step
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    status = co_alibi_attn.device_status(reset=True)

    # ---------------- the same K steps again with CUDA events around every kernel launch
    # (the backward then goes out as its three kernels, one C call each): per-kernel
    # times for the breakdown and the roofline
    impl.kernel_events = {}
    barrier()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(args.steps):
        step()
    g1.record()
    torch.cuda.synchronize()
    rec = impl.kernel_events
    impl.kernel_events = None
    ms_instr = g0.elapsed_time(g1) / args.steps
    kern_ms = {name: statistics.mean(a.elapsed_time(b) for a, b in pairs) for name, pairs in rec.items()}
    status = max(status, co_alibi_attn.device_status(reset=True))

    t = torch.tensor([ms, host_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, host_ms_max = t[0].item(), t[1].item()
    value = world * flops_step / (ms_max * 1e-3) / 1e12

    # ---------------- forward-only timing (the metric's fwd half)
    fwd_ms = kern_ms.get("fwd")
    # ---------------- e2e: pinned host inputs -> device -> API -> host outputs
    # through co_alibi_attention_from_host: batch elements streamed over three CUDA
    # streams (copy-in, kernels, copy-out overlap); every step copies its inputs in
    # and its results out, and returns with the results in host memory
    from co_alibi_attn.streaming import co_alibi_attention_from_host
    outs_h = [torch.empty_like(q_h).pin_memory()]
    if not fwd_only:
        outs_h += [torch.empty_like(q_h).pin_memory(), torch.empty_like(k_h).pin_memory(),
                   torch.empty_like(v_h).pin_memory()]

    e2e_slopes = (shard_slopes(Hq, shard, 8.0, dtype, dev) if args.scaling == "strong" and world > 1 else None)

    def e2e_step():
        co_alibi_attention_from_host(q_h, k_h, v_h, None if fwd_only else do_h, causal=causal, out=outs_h, device=dev,
                                     slopes=e2e_slopes)

    e2e_ms = float("nan")
    if args.e2e_steps > 0:
        e2e_step()
        torch.cuda.synchronize()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        f1.record()
        torch.cuda.synchronize()
        e2e_ms = f0.elapsed_time(f1) / args.e2e_steps
    t = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = t.item()
    h2d = sum(x.numel() * x.element_size() for x in ([q_h, k_h, v_h] + ([] if fwd_only else [do_h])))
    d2h = sum(x.numel() * x.element_size() for x in outs_h)
    copy_ms = pcie_copy_floor_ms([q_h, k_h, v_h] + ([] if fwd_only else [do_h]), outs_h, dev)

    # ---------------- roofline of the dominant kernel
    burst, sustained, hbm, peak_src = load_peaks()
    # which backward the library runs for this rank's problem: stored P / dS (pass B a
    # streaming GEMM, 4 D per score, no MUFU) or recompute (pass B 8 D and the maths)
    from co_alibi_attn import _lib as clib
    lib = clib.load()
    bargs = clib.CoalibiBwdArgs(B=B_r, Hq=Hq_r, Hkv=Hkv_r, Sq=S, Skv=S, D=D, causal=1 if causal else 0)
    stored = lib.coalibi_bwd_workspace_size(bargs) != lib.coalibi_bwd_workspace_min_bytes(B_r, Hq_r, Hkv_r, S, S, D)
    n_t = (S + 127) // 128
    tiles = B_r * Hq_r * (n_t * (n_t + 1) // 2 if causal else n_t * n_t)
    per_kernel_flops = {"fwd": 4.0 * D * E, "bwd_a": 6.0 * D * E, "bwd_b": (4.0 if stored else 8.0) * D * E,
                        "bwd_delta": 0.0}
    # MUFU ops per visible score: tanh sigmoid + exp2, less the quarter of the exp2
    # that the forward and the recompute path's D=128 pass B run as a polynomial on the FMA pipe
    mufu_b = 0.0 if stored else (1.75 if D == 128 else 2.0)
    per_kernel_mufu = {"fwd": 1.75 * E, "bwd_a": 2.0 * E, "bwd_b": mufu_b * E, "bwd_delta": 0.0}
    dom = max(kern_ms, key=kern_ms.get)
    ach = per_kernel_flops[dom] / (kern_ms[dom] * 1e-3) / 1e12
    sm_mhz = clocks["sm_mhz"] if clocks else 1965.0
    kernels = {}
    for name, kms in kern_ms.items():
        d = {"ms": round(kms, 4), "share": round(kms / ms_instr, 4)}
        if per_kernel_flops[name]:
            d["tflops"] = round(per_kernel_flops[name] / (kms * 1e-3) / 1e12, 2)
            d["mufu_frac"] = round(per_kernel_mufu[name] / (16 * 148 * sm_mhz * 1e6 * kms * 1e-3), 4)
        if name == "bwd_b" and stored:
            # its bound: the P and dS tiles pass A wrote, read once from HBM (Q / dO re-reads hit L2)
            pds = 2.0 * tiles * 128 * 128 * 2
            d["pds_read_gbs"] = round(pds / (kms * 1e-3) / 1e9, 1)
            d["hbm_frac"] = round(pds / (kms * 1e-3) / 1e9 / hbm, 4)
        kernels[name] = d
    roof = {"bound": "tensor", "kernel": dom, "achieved": round(ach, 2), "peak": burst, "unit": "TFLOP/s",
            "frac": round(ach / burst, 4), "peak_source": f"{peak_src} bf16_tflops (burst)",
            "traffic": NCU_TRAFFIC_CFG2.get(dom) if args.config == "cfg2" and B_r * Hkv_r == 8 * 16 else None,
            "flops_per_launch": per_kernel_flops[dom],
            "backward_path": "stored P / dS" if stored else "recompute",
            "note": "algorithmic FLOPs on causal-visible scores of the kernel's GEMMs "
                    "(fwd 4D, pass A 6D, pass B 4D stored path / 8D recompute path per score) / mean CUDA-event "
                    "duration in the kernel-timing pass (the timed region's K steps repeated with events around "
                    "each launch); second roofline: mufu_frac = MUFU ops per score (tanh + ex2 = 2, 1.75 where a "
                    "quarter of the ex2 is a polynomial) / (16 ops/clk/SM x 148 SMs x sampled clock)"}

    verification = None
    if not args.no_verify:
        verification = verify_shards(cfg, shard, world, rank, dev, q, k, v, do, attn)

    side = ref_triton = None
    if world == 1 and not args.no_side_by_side:
        with torch.no_grad():
            o_ours = co_alibi_attention(q, k, v, causal=causal).cpu()
        torch.cuda.synchronize()
        ref_triton = reference_triton_side_by_side(args, cfg, o_ours, ms_max, fwd_ms)
        del o_ours
        side = flash_side_by_side(cfg, dev, max(3, min(args.steps, 50)), args.warmup)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tfl, tsec, nth, desc = cpu_sample_tflops(cfg, S, 3)
        cpu = {"value": round(tfl, 6), "unit": "TFLOP/s", "cores": nth, "kind": "port", "sample": desc,
               "seconds_per_sample": round(tsec, 3)}

    if rank == 0:
        line = {
            "metric": metric_name(args.config), "value": round(value, 3), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": {torch.float16: "fp16", torch.bfloat16: "bf16"}[dtype],
            "data": "synthetic", "config": config_dict(args, cfg),
            "fwd_ms": round(fwd_ms, 4) if fwd_ms else None,
            "fwd_tflops": round(flops_fwd / (fwd_ms * 1e-3) / 1e12, 3) if fwd_ms else None,
            "fwd_pct_of_tensor_peak_spec2250": round(100 * flops_fwd / (fwd_ms * 1e-3) / 2.25e15, 2) if fwd_ms else None,
            "fwd_bwd_pct_of_tensor_peak_spec2250": round(100 * value / world / 2250.0, 2),
            "fwd_bwd_tflops_reference_convention": round(
                world * (12.0 * D * S * S * B_r * Hq_r if not fwd_only else 4.0 * D * S * S * B_r * Hq_r)
                / (ms_max * 1e-3) / 1e12, 3),
            "host_enqueue_ms_per_step": round(host_ms_max, 4),
            "kernels": kernels, "kernel_timing_pass_ms_per_step": round(ms_instr, 4),
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(world * flops_step / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "copy_only_ms": round(copy_ms, 3),
                    "copy_only_frac": round(copy_ms / e2e_ms, 4),
                    "note": "copy_only_ms: the same bytes copied host->device and device->host at once (pinned "
                            "buffers, two streams, no kernels); e2e can be no faster"},
            "gpu_launches": kernels_per_step * args.steps, "clocks": clocks, "device_status": status,
            "verification": verification,
            "reference_triton": ref_triton,
            "side_by_side": side,
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
