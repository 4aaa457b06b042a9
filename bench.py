#!/usr/bin/env python3
"""Benchmark of the bitgpu attention hot path on B200.

Headline (BASELINE.json metric "decode-attn HBM GB/s (% peak) @32K ctx, q8/f16 KV; prefill-attn
TFLOP/s"), measured on config 2: Qwen3-8B-shape batched decode attention, 32 Q / 8 KV heads,
head_dim 128, batch 64 sequences per GPU, 32768 cached positions each, one query token, f16 KV
cache (the q8 cache is measured in the same run under "variants").  A step = one layer of
decode attention over the whole batch with the cache resident in HBM (8.59 GB f16, far larger
than the 126 MB L2, so no flush is needed between steps).

Arms:
  python bench.py [--gpus N --steps K --warmup W]     the B200 kernels (this repo)
  python bench.py --impl reference ...                 the reference's CPU path (numpy port of
                                                       tools/reference.py attention + the WGSL
                                                       f16 read), timed on the host cores
Multi-GPU: launched by torch.distributed.run; every rank runs its own batch of 64 (weak scaling,
batch-sharded, no communication); the step time is the max over ranks.
"""
import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# config 2; manifest models/bonsai-8b-gguf: heads 32, kv_heads 8, head_dim 128
B, L, H, KV, D = 64, 32768, 32, 8, 128
ROW_BYTES = {"f16": D * 2, "q8": D + (D // 32) * 4, "q8r": D + 4, "f32": D * 4}


def alg_bytes(mode, batch=B, ctx=L):
    """Algorithmic bytes of one decode step: every cached K and V row read once, q read and the
    f32 output written once per head."""
    return batch * 2 * ctx * KV * ROW_BYTES[mode] + batch * 2 * H * D * 4


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=B, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--modes", default="f16,q8", help="KV modes to run (the first is the headline)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill"],
                    help="decode: config 2 headline (+ prefill variant); prefill: config 3 alone")
    ap.add_argument("--seq", type=int, default=8192, help="prefill tokens per sequence (config 3: 8192)")
    ap.add_argument("--prefill-batch", type=int, default=8, help="prefill sequences per GPU (config 3: 8)")
    ap.add_argument("--no-prefill", action="store_true")
    return ap.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def peaks():
    try:
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock / throttle-reason sampler running during the timed region (NVML every 5 ms;
    the same fields as the nvidia-smi clocks query)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        import threading
        self.samples, self.err = [], None
        self.stop_ev = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[index]) if vis and vis.split(",")[index].isdigit() else index
            self.h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.nv = pynvml
            self.max = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self.err = f"nvml unavailable: {e}"
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((sm, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def stop(self):
        if self.err:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err]}
        self.stop_ev.set()
        self.t.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": ["no samples"]}
        sm = [x[0] for x in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        loaded = [x for x in sm if x > 0.5 * self.max] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": self.max, "samples": len(sm),
                "sm_mhz_min": min(sm), "reasons": reasons, "source": "nvml, 5 ms"}


def make_cache(ops, torch, mode, seed, batch=B, ctx=L):
    """Fill a cache with seeded N(0,1) K/V through the library's own append (the codec)."""
    cache = ops.KVCache(batch, ctx, KV, D, mode=mode, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    chunk = 2048
    for p0 in range(0, ctx, chunk):
        n = min(chunk, ctx - p0)
        for which in (0, 1):
            x = torch.randn((batch, n, KV, D), generator=g, device="cuda", dtype=torch.float32)
            cache.append(which, x, p0)
    torch.cuda.synchronize()
    return cache


def time_steps(torch, fn, steps, warmup, barrier):
    for _ in range(warmup):
        fn()
    barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps  # ms per step


def cpu_baseline(mode, seconds, seed=0):
    """The oracle (numpy port of the reference attention, f32 math over the storage codec's
    values) on one sequence x one layer of config 2, repeated for ~`seconds`."""
    import numpy as np
    from oracle import attention as OA
    from oracle import kvcodec
    rng = np.random.default_rng(seed)
    kr = rng.standard_normal((L, KV, D), dtype=np.float32)
    vr = rng.standard_normal((L, KV, D), dtype=np.float32)
    kd = kvcodec.decode(mode, *kvcodec.encode(mode, kr))
    vd = kvcodec.decode(mode, *kvcodec.encode(mode, vr))
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    OA.attend(q, kd, vd, L - 1)
    n, t0 = 0, time.perf_counter()
    while True:
        OA.attend(q, kd, vd, L - 1)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    per = el / n
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        cores = os.cpu_count()
    gbs = alg_bytes(mode, batch=1) / per / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"oracle numpy attention, 1 sequence x 1 layer of config 2 ({mode} cache, ctx {L}), "
                      f"{n} reps in {el:.1f} s; same algorithmic bytes per sequence as the GPU metric",
            "ms_per_sequence": round(per * 1e3, 3)}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np
    from oracle import attention as OA
    from oracle import kvcodec
    rng = np.random.default_rng(0)
    kr = rng.standard_normal((L, KV, D), dtype=np.float32)
    vr = rng.standard_normal((L, KV, D), dtype=np.float32)
    kd = kvcodec.decode("f16", *kvcodec.encode("f16", kr))
    vd = kvcodec.decode("f16", *kvcodec.encode("f16", vr))
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    for _ in range(args.warmup):
        OA.attend(q, kd, vd, L - 1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        OA.attend(q, kd, vd, L - 1)
    per = (time.perf_counter() - t0) / args.steps
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        cores = os.cpu_count()
    val = alg_bytes("f16", batch=1) / per / 1e9
    sample = (f"one sequence x one layer of config 2 per step (f16 cache, ctx {L}); the reference's CPU attention "
              f"path restated in numpy (oracle/attention.py), {cores} BLAS threads")
    line = {"metric": METRIC, "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seed 0",
            "config": CONFIG,
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


METRIC = "decode-attn HBM GB/s @32K ctx (config 2, Qwen3-8B shape, f16 KV)"
CONFIG = {"workload": "config 2: batched decode attention, Qwen3-8B shape (H32 KV8 D128), batch 64 per GPU, "
                      "ctx 32768, S=1, f16 KV cache, one layer per step",
          "global_batch_per_gpu": B, "seq_len": L, "l2": "cache 8.59 GB per GPU >> 126 MB L2; no flush needed",
          "parallelism": "batch-sharded, no communication"}


def profiled_traffic(mode, batch):
    """DRAM traffic per launch of the decode kernel from the committed ncu summary
    (profiles/attn_tc_decode_<mode>.md, line `traffic_bytes_per_sequence = N`), scaled to `batch`
    sequences (traffic grows linearly with the sequences a launch processes), or None."""
    try:
        for line in open(os.path.join(ROOT, "profiles", f"attn_tc_decode_{mode}.md")):
            if line.strip().startswith("traffic_bytes_per_sequence"):
                return int(float(line.split("=")[1].strip().split()[0]) * batch)
    except OSError:
        pass
    return None


# config 3; manifest models/bonsai-4b-gguf: heads 32, kv_heads 8, head_dim 128
PF_H, PF_KV = 32, 8


def prefill_flops(batch, seq):
    """QK^T and PV over the causal half including the diagonal, 2 flop per MAC."""
    return 4.0 * D * PF_H * batch * seq * (seq + 1) / 2


def run_prefill(torch, ops, args, rank, barrier, max_over_ranks, clocks_for=None):
    """Config 3: causal prefill attention of `batch` x `seq` f16 tokens over the f16 cache those
    tokens were appended to (posBase 0), f16 output; then the step's K/V rows written into an f16
    and a q8 cache (timed separately, as bytes)."""
    nb, S = args.prefill_batch, args.seq
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    k16 = torch.randn((nb, S, PF_KV, D), generator=g, device="cuda").half()
    v16 = torch.randn((nb, S, PF_KV, D), generator=g, device="cuda").half()
    cache = ops.KVCache(nb, S, PF_KV, D, mode="f16", device="cuda")
    cache.append(0, k16, 0)
    cache.append(1, v16, 0)
    q = torch.randn((nb, S, PF_H, D), generator=g, device="cuda").half()
    out = torch.empty((nb, S, PF_H, D), device="cuda", dtype=torch.float16)
    clk = Clocks(clocks_for) if clocks_for is not None else None
    ms = max_over_ranks(time_steps(torch, lambda: ops.attention(q, cache, 0, out=out), args.steps, args.warmup,
                                   barrier))
    res = {"ms": ms, "flops": prefill_flops(nb, S)}
    if clk:
        res["clocks"] = clk.stop()
    # the prefill's K/V written into an f16 cache and a q8 cache (kv append, HBM-bound)
    c16 = ops.KVCache(nb, S, PF_KV, D, mode="f16", device="cuda")
    c8 = ops.KVCache(nb, S, PF_KV, D, mode="q8", device="cuda")

    def writes():
        for c in (c16, c8):
            c.append(0, k16, 0)
            c.append(1, v16, 0)
    wms = max_over_ranks(time_steps(torch, writes, max(3, args.steps // 4), 2, barrier))
    wbytes = 2 * k16.numel() * 2 * 2 + 2 * k16.numel() * (2 + 1) + 2 * (k16.numel() // 32) * 4
    res["kv_write"] = {"ms": round(wms, 4), "GB/s": round(wbytes / (wms * 1e-3) / 1e9, 1),
                       "bytes": wbytes, "note": "K and V of the prefill into an f16 and a q8 cache"}
    del cache, c16, c8, q, out
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl")
    barrier = (lambda: dist.barrier()) if dist else (lambda: None)
    from bitgpu_b200 import ops
    hbm, _, peak_kind = peaks()
    nb = args.batch
    modes = [m for m in args.modes.split(",") if m]

    def max_over_ranks(ms):
        if not dist:
            return ms
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    _, bf16_peak, _ = peaks()
    if args.workload == "prefill":
        r = run_prefill(torch, ops, args, rank, barrier, max_over_ranks, clocks_for=local)
        if rank == 0:
            tf = r["flops"] * ws / (r["ms"] * 1e-3) / 1e12
            per = r["flops"] / (r["ms"] * 1e-3) / 1e12
            print(json.dumps({
                "metric": "prefill-attn TFLOP/s (config 3, Qwen3-4B shape, causal, f16)", "value": round(tf, 2),
                "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(r["ms"], 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic N(0,1), seeded",
                "config": {"workload": f"config 3: causal prefill, H32 KV8 D128, batch {args.prefill_batch}, "
                                       f"seq {args.seq}, f16 Q/K/V, f32 accumulate, f16 out",
                           "l2": "Q+K/V+out >> 126 MB L2"},
                "roofline": {"bound": "tensor", "achieved": round(per, 1), "peak": bf16_peak, "unit": "TFLOP/s",
                             "frac": round(per / bf16_peak, 4), "peak_kind": "measured cuBLAS bf16 burst",
                             "traffic": None},
                "gpu_launches": args.steps, "clocks": r.get("clocks"), "kv_write": r["kv_write"]}), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    q = torch.randn((nb, 1, H, D), device="cuda", generator=torch.Generator(device="cuda").manual_seed(100 + rank))
    results = {}
    for i, mode in enumerate(modes):
        cache = make_cache(ops, torch, mode, seed=1000 * rank + i + 1, batch=nb)
        out = torch.empty((nb, 1, H, D), device="cuda")
        fn = lambda: ops.attention(q, cache, L - 1, out=out)
        clk = Clocks(local) if i == 0 else None
        ms = max_over_ranks(time_steps(torch, fn, args.steps, args.warmup, barrier))
        ab = alg_bytes(mode, batch=nb)
        res = {"ms": ms, "gbs": ab * ws / (ms * 1e-3) / 1e9, "per_gpu_gbs": ab / (ms * 1e-3) / 1e9, "bytes": ab}
        if i == 0:
            res["clocks"] = clk.stop()
        if i == 0 and not args.no_e2e:
            # e2e through the public API: pinned host q + the step's new K/V rows in, the attention
            # output back out, every step (the cache itself stays resident, as in the engine)
            qh = torch.randn((nb, 1, H, D)).pin_memory()
            kh = torch.randn((nb, 1, KV, D)).pin_memory()
            vh = torch.randn((nb, 1, KV, D)).pin_memory()
            oh = torch.empty((nb, 1, H, D)).pin_memory()
            qd = torch.empty_like(q)
            kd = torch.empty((nb, 1, KV, D), device="cuda")
            vd = torch.empty((nb, 1, KV, D), device="cuda")

            def e2e():
                qd.copy_(qh, non_blocking=True)
                kd.copy_(kh, non_blocking=True)
                vd.copy_(vh, non_blocking=True)
                cache.append(0, kd, L - 1)
                cache.append(1, vd, L - 1)
                ops.attention(qd, cache, L - 1, out=out)
                oh.copy_(out, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                float(oh[0, 0, 0, 0])     # the host reads the step's result
            ms_e2e = max_over_ranks(time_steps(torch, e2e, args.steps, args.warmup, barrier))
            res["e2e"] = {"value": round(ab * ws / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                          "h2d_bytes_per_step": (qh.numel() + kh.numel() + vh.numel()) * 4,
                          "d2h_bytes_per_step": oh.numel() * 4, "ms_per_step": round(ms_e2e, 4),
                          "path": "bitgpu_b200.ops (ctypes -> libbgattn.so C ABI): bg_kv_append x2 + bg_attention"}
        results[mode] = res
        del cache
        torch.cuda.empty_cache()
    pf = None
    if not args.no_prefill:
        pa = argparse.Namespace(**vars(args))
        pa.steps, pa.warmup = max(3, min(args.steps, 20)), 3
        pf = run_prefill(torch, ops, pa, rank, barrier, max_over_ranks)

    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    head = results[modes[0]]
    per_launch = head["bytes"] / (head["ms"] * 1e-3) / 1e9
    traffic = profiled_traffic(modes[0], nb)
    line = {
        "metric": METRIC, "value": round(head["gbs"], 2), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(head["ms"], 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": modes[0],
        "data": "synthetic N(0,1), seeded; KV written through the library's own f16/q8 append",
        "config": dict(CONFIG, global_batch_per_gpu=nb, kv_mode=modes[0]),
        "roofline": {"bound": "hbm", "achieved": round(per_launch, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(per_launch / hbm, 4), "peak_kind": f"{peak_kind} (copy, read+write)",
                     "traffic": traffic, "algorithmic_bytes": head["bytes"],
                     "note": "achieved = algorithmic bytes per launch (2*B*L*KV*rowB + 2*B*H*D*4) / mean duration "
                             "of one bg_attention call (split-KV kernel + LSE merge), CUDA events on its stream; "
                             "traffic = ncu dram read+write bytes per sequence (profiles/) x batch"},
        "gpu_launches": 2 * args.steps,
        "clocks": head["clocks"],
        "variants": {m: {"value": round(r["gbs"], 2), "unit": "GB/s", "ms_per_step": round(r["ms"], 4),
                         "frac": round(r["per_gpu_gbs"] / hbm, 4), "bytes_per_step_per_gpu": r["bytes"]}
                     for m, r in results.items() if m != modes[0]},
    }
    if pf:
        tf = pf["flops"] / (pf["ms"] * 1e-3) / 1e12
        line["variants"]["prefill"] = {
            "metric": "prefill-attn TFLOP/s (config 3)", "value": round(tf * ws, 2), "unit": "TFLOP/s",
            "ms_per_step": round(pf["ms"], 4), "frac": round(tf / bf16_peak, 4),
            "peak": bf16_peak, "peak_kind": "measured cuBLAS bf16 burst", "flops_per_step_per_gpu": pf["flops"],
            "kv_write": pf["kv_write"]}
    if "e2e" in head:
        line["e2e"] = head["e2e"]
    if ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(modes[0], args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
