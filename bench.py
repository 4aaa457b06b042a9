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
# NCCL's INIT lines (rank count, transport, NVLS) go to stderr: stdout carries only the JSON line
os.environ.setdefault("NCCL_DEBUG", "INFO")
os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

# config 2; manifest models/bonsai-8b-gguf: heads 32, kv_heads 8, head_dim 128
B, L, H, KV, D = 64, 32768, 32, 8, 128
GA_L_DEFAULT = 131072
ROW_BYTES = {"f16": D * 2, "q8": D + (D // 32) * 4, "q8r": D + 4, "f32": D * 4}


def alg_bytes(mode, batch=B, ctx=L):
    """Algorithmic bytes of one decode step: every cached K and V row read once, q read and the
    f32 output written once per head."""
    return batch * 2 * ctx * KV * ROW_BYTES[mode] + batch * 2 * H * D * 4


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=B, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--modes", default="f16,q8", help="KV modes to run (the first is the headline)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "gated", "deltanet", "roll"],
                    help="decode: config 2 headline (+ the other configs as variants); others: one config alone")
    ap.add_argument("--gated-ctx", type=int, default=GA_L_DEFAULT)
    ap.add_argument("--dn-prefill", type=int, default=4096)
    ap.add_argument("--roll-batch", type=int, default=32)
    ap.add_argument("--roll-steps", type=int, default=2048)
    ap.add_argument("--variants", default="q8,prefill,gated,deltanet,roll",
                    help="configs measured as variants of the default decode run")
    ap.add_argument("--seq", type=int, default=8192, help="prefill tokens per sequence (config 3: 8192)")
    ap.add_argument("--prefill-batch", type=int, default=8, help="prefill sequences per GPU (config 3: 8)")
    ap.add_argument("--prefill-cache", default="f16", choices=["f16", "q8", "f32"],
                    help="--workload prefill: cache codec (q8: the engine's 8-bit cache; f32: 3xTF32 kernel)")
    ap.add_argument("--prefill-q", default="f16", choices=["f16", "f32"], help="--workload prefill: query dtype")

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


def host_threads():
    """Use every host core for the CPU arms (torch.distributed.run sets OMP_NUM_THREADS=1 for
    each rank, which would otherwise leave the numpy reference on one BLAS thread).  Returns
    (threads used, physical cores, logical cores)."""
    logical = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    try:
        import psutil
        physical = psutil.cpu_count(logical=False) or logical
    except Exception:  # noqa: BLE001
        physical = logical
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=physical)
    except Exception:  # noqa: BLE001
        pass
    try:
        from threadpoolctl import threadpool_info
        used = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001
        used = physical
    return used, physical, logical


def cpu_baseline(mode, seconds, seed=0):
    """The oracle (numpy port of the reference attention, f32 math over the storage codec's
    values) on one sequence x one layer of config 2, repeated for ~`seconds`."""
    import numpy as np
    from oracle import attention as OA
    from oracle import kvcodec
    host_threads()
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
    cores, physical, logical = host_threads()
    gbs = alg_bytes(mode, batch=1) / per / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "physical_cores": physical,
            "logical_cores": logical, "kind": "port",
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
    cores, physical, logical = host_threads()
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
    val = alg_bytes("f16", batch=1) / per / 1e9
    sample = (f"one sequence x one layer of config 2 per step (f16 cache, ctx {L}); the reference's CPU attention "
              f"path restated in numpy (oracle/attention.py), {cores} BLAS threads")
    line = {"metric": METRIC, "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic N(0,1), seed 0",
            "config": dict(CONFIG, global_batch_per_gpu=B, kv_mode="f16"),
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": cores, "physical_cores": physical,
                             "logical_cores": logical, "kind": "port", "sample": sample},
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


def tf32_peak(torch, n=8192, reps=10):
    """Dense TF32 tensor-core throughput measured here: torch.matmul of two n x n f32 matrices
    with TF32 allowed (cuBLAS), best of `reps`, 2*n^3 flops per product."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn((n, n), device="cuda")
        b = torch.randn((n, n), device="cuda")
        c = a @ b
        best = None
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        del a, b, c
        torch.cuda.empty_cache()
        return {"tflops": round(2.0 * n ** 3 / (best * 1e-3) / 1e12, 1), "how": f"cuBLAS TF32 matmul {n}^3, best of {reps}"}
    except Exception as e:  # noqa: BLE001
        return {"tflops": None, "how": f"unavailable: {e}"}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def run_prefill(torch, ops, args, rank, barrier, max_over_ranks, clocks_for=None, mode="f16", q32=False,
                kv_write=True):
    """Config 3: causal prefill attention of `batch` x `seq` tokens over the cache those tokens
    were appended to (posBase 0), f16 output.  Default: f16 queries over an f16 cache (BASELINE's
    wording); mode="q8", q32=True is the engine's own call (f32 queries over the 8-bit cache,
    engine.ts:1580).  Then the step's K/V rows written into an f16 and a q8 cache (timed
    separately, as bytes)."""
    nb, S = args.prefill_batch, args.seq
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    k16 = torch.randn((nb, S, PF_KV, D), generator=g, device="cuda").half()
    v16 = torch.randn((nb, S, PF_KV, D), generator=g, device="cuda").half()
    cache = ops.KVCache(nb, S, PF_KV, D, mode=mode, device="cuda")
    cache.append(0, k16, 0)
    cache.append(1, v16, 0)
    q = torch.randn((nb, S, PF_H, D), generator=g, device="cuda")
    if not q32:
        q = q.half()
    out = torch.empty((nb, S, PF_H, D), device="cuda", dtype=torch.float16)
    clk = Clocks(clocks_for) if clocks_for is not None else None
    ms = max_over_ranks(time_steps(torch, lambda: ops.attention(q, cache, 0, out=out), args.steps, args.warmup,
                                   barrier))
    res = {"ms": ms, "flops": prefill_flops(nb, S)}
    if clk:
        res["clocks"] = clk.stop()
    if not kv_write:
        del cache, q, out
        torch.cuda.empty_cache()
        return res
    # the prefill's K/V written into an f16 cache and a q8 cache (kv append, HBM-bound)
    c16 = ops.KVCache(nb, S, PF_KV, D, mode="f16", device="cuda")
    c8 = ops.KVCache(nb, S, PF_KV, D, mode="q8", device="cuda")

    def writes():
        c16.append_kv_pair(c8, k16, v16, 0)   # one pass: source read once, both caches written
    wms = max_over_ranks(time_steps(torch, writes, max(3, args.steps // 4), 2, barrier))
    # f16 K/V read once; f16 cache rows + q8 codes + q8 block scales written
    wbytes = 2 * k16.numel() * 2 + 2 * k16.numel() * (2 + 1) + 2 * (k16.numel() // 32) * 4
    res["kv_write"] = {"ms": round(wms, 4), "GB/s": round(wbytes / (wms * 1e-3) / 1e9, 1), "bytes": wbytes,
                       "note": "K and V of the prefill into an f16 and a q8 cache in one pass (bg_kv_append_kv_pair)"}
    del cache, c16, c8, q, out
    torch.cuda.empty_cache()
    return res


# config 5b; manifest models/bonsai-27b-gguf: heads 24, kv_heads 4, head_dim 256
GA_H, GA_KV, GA_D, GA_L = 24, 4, 256, 131072


def run_gated(torch, ops, args, ws, rank, barrier, max_over_ranks):
    """Config 5b: one stream's gated head_dim-256 decode at 131072 positions, the cache split over
    the ranks (bitgpu_b200.splitkv: split-KV partials pushed into every rank over NVLink, merge with
    the gate fused; the NCCL all-gather form timed beside it)."""
    from bitgpu_b200.splitkv import SplitKVDecoder
    L = args.gated_ctx
    dec = SplitKVDecoder(L)
    n = dec.hi - dec.lo
    g = torch.Generator(device="cuda").manual_seed(11 + rank)
    cache = ops.KVCache(1, n, GA_KV, GA_D, mode="f16", device="cuda")
    for p0 in range(0, n, 8192):
        m = min(8192, n - p0)
        for w in (0, 1):
            cache.append(w, torch.randn((1, m, GA_KV, GA_D), generator=g, device="cuda"), p0)
    gq = torch.Generator(device="cuda").manual_seed(12)          # identical q / gate on every rank
    q = torch.randn((1, 1, GA_H, GA_D), generator=gq, device="cuda")
    gate = torch.randn((1, 1, GA_H, GA_D), generator=gq, device="cuda")
    scale = 1.0 / GA_D ** 0.5
    byts = 2 * L * GA_KV * GA_D * 2 + 3 * GA_H * GA_D * 4
    if ws == 1:
        out = torch.empty_like(q)
        fn = lambda: ops.attention(q, cache, L - 1, scale=scale, gate=gate, out=out)
        launches = 1
    else:
        # the whole step -- split-KV kernel, push of the rows into every rank's gather buffer over
        # NVLink, merge -- replayed as one CUDA graph, so the host adds nothing per step
        fn = ops.Graphed(lambda: dec.step(q, cache, L - 1, gate=gate, scale=scale))
        launches = 3
    ms = max_over_ranks(time_steps(torch, fn, args.steps, args.warmup, barrier))
    res = {"ms": ms, "bytes": byts, "gbs": byts / (ms * 1e-3) / 1e9, "launches_per_step": launches,
           "exchange": dec.exchange if ws > 1 else None,
           "exchange_bytes_per_rank": 0 if ws == 1 else GA_H * (GA_D + 2) * 4 * ws}
    if ws > 1:
        # the same step with the NCCL all-gather exchange (A/B)
        dn = SplitKVDecoder(L, exchange="nccl")
        fn2 = ops.Graphed(lambda: dn.step(q, cache, L - 1, gate=gate, scale=scale))
        res["nccl_ms"] = max_over_ranks(time_steps(torch, fn2, args.steps, args.warmup, barrier))
        # strong scaling of this config: the whole 131072-position step on one GPU (rank 0)
        del cache
        torch.cuda.empty_cache()
        one = 0.0
        if rank == 0:
            full = ops.KVCache(1, L, GA_KV, GA_D, mode="f16", device="cuda")
            for p0 in range(0, L, 8192):
                m = min(8192, L - p0)
                for w in (0, 1):
                    full.append(w, torch.randn((1, m, GA_KV, GA_D), generator=g, device="cuda"), p0)
            out1 = torch.empty_like(q)
            one = time_steps(torch, lambda: ops.attention(q, full, L - 1, scale=scale, gate=gate, out=out1),
                             args.steps, args.warmup, lambda: None)
            del full
            torch.cuda.empty_cache()
        barrier()
        res["ms_1gpu"] = max_over_ranks(one)
        res["strong_scaling_efficiency"] = res["ms_1gpu"] / (ws * ms)
        del fn, fn2
        dec.close()
        dn.close()
    else:
        del cache
        torch.cuda.empty_cache()
    return res


# config 5a; 27B hybrid linear layer: 16 key heads, 48 value heads, 128 x 128
DN_HK, DN_H, DN_DK, DN_DV = 16, 48, 128, 128


def deltanet_decode_bytes():
    """Per decode token: the f32 state in and out, q/k of the key heads, v/z/output of the value
    heads, a/b gate inputs."""
    return 2 * DN_H * DN_DK * DN_DV * 4 + (2 * DN_HK * DN_DK + 3 * DN_H * DN_DV + 2 * DN_H) * 4


DN_LAYERS = 48  # linear (DeltaNet) layers of the 27B hybrid, one decode token through all of them


def run_deltanet(torch, ops, args, rank, barrier, max_over_ranks):
    """Config 5a: a 4096-token gated-DeltaNet prefill (g/beta -> recurrence -> gated norm, one
    fused launch) and then single-token decode steps continuing its state.  B=1 is one sequential
    scan: multi-GPU runs are independent replicas."""
    S = args.dn_prefill
    g = torch.Generator(device="cuda").manual_seed(21 + rank)
    r = lambda *sh: torch.randn(sh, generator=g, device="cuda")
    q, k, v, z = r(S, DN_HK, DN_DK), r(S, DN_HK, DN_DK), r(S, DN_H, DN_DV), r(S, DN_H, DN_DV)
    a, b = r(S, DN_H), r(S, DN_H)
    a_neg, dt = -torch.ones(DN_H, device="cuda"), torch.zeros(DN_H, device="cuda")
    gamma = torch.ones(DN_DV, device="cuda")
    st = torch.zeros((DN_H, DN_DK, DN_DV), device="cuda")
    pf_rec = lambda: ops.deltanet_fused(q, k, v, a, b, a_neg, dt, z, gamma, 1e-6, state_in=None, state_out=st)
    ms_rec = max_over_ranks(time_steps(torch, pf_rec, max(3, args.steps // 10), 3, barrier))
    pf = lambda: ops.deltanet_chunked(q, k, v, a, b, a_neg, dt, z, gamma, 1e-6, state_in=None, state_out=st)
    ms_pf = max_over_ranks(time_steps(torch, pf, max(3, args.steps // 5), 3, barrier))
    # One decode token through DN_LAYERS linear layers (the 27B's 48), each with its own state,
    # captured as one CUDA graph: the per-layer kernels run back to back as in an engine's stream,
    # and the 151 MB of states exceed the 126 MB L2, so every layer streams its state from HBM.
    states = torch.zeros((DN_LAYERS, DN_H, DN_DK, DN_DV), device="cuda")
    states[0].copy_(st)

    def dec_layers():
        for li in range(DN_LAYERS):
            t = li % S
            ops.deltanet_fused(q[t:t + 1], k[t:t + 1], v[t:t + 1], a[t:t + 1], b[t:t + 1], a_neg, dt, z[t:t + 1],
                               gamma, 1e-6, state_in=states[li], state_out=states[li])
    dec = ops.Graphed(dec_layers)
    ms_dec = max_over_ranks(time_steps(torch, dec, args.steps, args.warmup, barrier)) / DN_LAYERS
    flops_pf = S * DN_H * 4 * DN_DK * DN_DV * 2
    return {"prefill_ms": ms_pf, "prefill_recurrent_ms": ms_rec, "prefill_tokens": S, "prefill_tflops": flops_pf / (ms_pf * 1e-3) / 1e12,
            "decode_ms": ms_dec, "decode_bytes": deltanet_decode_bytes(),
            "decode_gbs": deltanet_decode_bytes() / (ms_dec * 1e-3) / 1e9}


# config 4; Qwen3-1.7B shape: 16 Q / 8 KV heads, head_dim 128
RL_H, RL_KV, RL_SINKS, RL_WINDOW = 16, 8, 4, 4096


def rope_tables(torch, positions, D, theta=1e6, factor=4.0, orig=8192):
    """YaRN rope tables [positions, D/2] in float64 angles, one float32 rounding (the reference's
    synthRope recipe; manifest bonsai-1.7b-gguf: theta 1e6, yarn factor 4, orig 8192)."""
    import math
    half = D // 2
    j = torch.arange(half, dtype=torch.float64)
    pf = theta ** (2 * j / D)
    lo = max(0, math.floor(D * math.log(orig / (32 * 2 * math.pi)) / (2 * math.log(theta))))
    hi = min(half - 1, math.ceil(D * math.log(orig / (2 * math.pi)) / (2 * math.log(theta))))
    ramp = ((j - lo) / (hi - lo)).clamp(0, 1)
    inv = (1 / (factor * pf)) * ramp + (1 / pf) * (1 - ramp)
    ms = float(torch.tensor(0.1 * math.log(factor) + 1, dtype=torch.float32))
    ang = torch.outer(torch.arange(positions, dtype=torch.float64), inv)
    return (torch.cos(ang) * ms).float().cuda(), (torch.sin(ang) * ms).float().cuda()


def run_roll(torch, ops, args, rank, barrier, max_over_ranks):
    """Config 4: sink-mode decode stream, batch 32, q8 ring of 4 sinks + 4096 slots.  Every step:
    evictFor (ring head advance when full), append the step's unroped K and V, attention with
    rope-at-read by logical slot.  Timed over `roll_steps` consecutive steps that cross
    evictions; the metric is mean algorithmic GB/s over those steps."""
    nb, maxlen = args.roll_batch, RL_SINKS + RL_WINDOW
    cache = ops.KVCache(nb, maxlen, RL_KV, D, mode="q8", sinks=RL_SINKS, window=RL_WINDOW, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(31 + rank)
    fill = maxlen - 1024                      # steady-state fill right after an eviction (3076)
    for p0 in range(0, fill, 1024):
        m = min(1024, fill - p0)
        for w in (0, 1):
            cache.append(w, torch.randn((nb, m, RL_KV, D), generator=g, device="cuda"), p0)
    cos_t, sin_t = rope_tables(torch, maxlen, D)
    T = args.roll_steps
    ks = torch.randn((T, nb, 1, RL_KV, D), generator=g, device="cuda")
    vs = torch.randn((T, nb, 1, RL_KV, D), generator=g, device="cuda")
    qs = torch.randn((T, nb, 1, RL_H, D), generator=g, device="cuda")
    out = torch.empty((nb, 1, RL_H, D), device="cuda")
    state = {"fill": fill, "t": 0, "bytes": 0}

    def step():
        t = state["t"] % T
        f = cache.evict_for(state["fill"], 1, maxlen)
        cache.append_kv(ks[t], vs[t], f)
        ops.attention(qs[t], cache, f, cos_t=cos_t, sin_t=sin_t, out=out)
        state["fill"] = f + 1
        state["t"] += 1
        state["bytes"] += nb * 2 * (f + 1) * RL_KV * (D + 16) + (f + 1) * (D // 2) * 8
    for _ in range(3):
        step()
    state["bytes"] = 0
    ms = time_steps(torch, step, T, 0, barrier)
    byts = state["bytes"] / T
    ms = max_over_ranks(ms)
    del cache
    torch.cuda.empty_cache()
    return {"ms": ms, "bytes_per_step": byts, "gbs": byts / (ms * 1e-3) / 1e9, "steps": T,
            "fill_range": [maxlen - 1024, maxlen], "ring_head": None}


def _base_line(args, ws, metric, value, unit, ms, dtype, config, roofline, launches, clocks=None):
    return {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic N(0,1), seeded", "config": config,
            "roofline": roofline, "gpu_launches": launches, "clocks": clocks}


def run_ours(args):
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
    barrier = (lambda: dist.barrier()) if dist else (lambda: None)
    from bitgpu_b200 import ops
    hbm, bf16_peak, peak_kind = peaks()
    nb = args.batch

    def max_over_ranks(ms):
        if not dist:
            return ms
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def finish(line):
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist:
            dist.destroy_process_group()

    def hbm_roof(gbs_per_gpu, note, traffic=None):
        return {"bound": "hbm", "achieved": round(gbs_per_gpu, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(gbs_per_gpu / hbm, 4), "peak_kind": f"{peak_kind} (copy, read+write)",
                "traffic": traffic, "note": note}

    # ---------------- single-config workloads ----------------
    if args.workload == "prefill":
        clk = Clocks(local)
        r = run_prefill(torch, ops, args, rank, barrier, max_over_ranks, mode=args.prefill_cache,
                        q32=args.prefill_q == "f32", kv_write=args.prefill_cache == "f16" and args.prefill_q == "f16")
        per = r["flops"] / (r["ms"] * 1e-3) / 1e12
        line = _base_line(args, ws, "prefill-attn TFLOP/s (config 3, Qwen3-4B shape, causal)", per * ws,
                          "TFLOP/s", r["ms"], "f16",
                          {"workload": f"config 3: causal prefill, H32 KV8 D128, batch {args.prefill_batch}, "
                                       f"seq {args.seq}, {args.prefill_q} Q over a {args.prefill_cache} cache, "
                                       f"f32 accumulate, f16 out",
                           "l2": "Q + K/V + out >> 126 MB L2"},
                          {"bound": "tensor", "achieved": round(per, 1), "peak": bf16_peak, "unit": "TFLOP/s",
                           "frac": round(per / bf16_peak, 4), "peak_kind": f"{peak_kind} cuBLAS bf16 burst",
                           "traffic": None}, args.steps, clk.stop())
        if "kv_write" in r:
            line["kv_write"] = r["kv_write"]
        return finish(line)
    if args.workload == "gated":
        clk = Clocks(local)
        r = run_gated(torch, ops, args, ws, rank, barrier, max_over_ranks)
        line = _base_line(args, ws, "gated decode-attn HBM GB/s (config 5b, 27B hybrid, D256, f16, split-KV)",
                          r["gbs"], "GB/s", r["ms"], "f16",
                          {"workload": f"config 5b: one stream, H24 KV4 D256, ctx {args.gated_ctx} f16, sigmoid "
                                       f"gate, KV positions split over {ws} GPU(s), NCCL all-gather + LSE merge",
                           "l2": "cache 537 MB >> 126 MB L2", "scaling_note": "fixed total work (strong)"},
                          hbm_roof(r["gbs"] / ws, "per-GPU share of the step's algorithmic bytes / step time"),
                          r["launches_per_step"] * args.steps, clk.stop())
        line["scaling"] = "strong"
        line["exchange"] = r["exchange"]
        line["exchange_bytes_per_rank_per_step"] = r["exchange_bytes_per_rank"]
        for k in ("nccl_ms", "ms_1gpu", "strong_scaling_efficiency"):
            if k in r:
                line[k] = round(r[k], 4)
        return finish(line)
    if args.workload == "deltanet":
        clk = Clocks(local)
        r = run_deltanet(torch, ops, args, rank, barrier, max_over_ranks)
        line = _base_line(args, ws, "deltanet decode HBM GB/s (config 5a, 27B hybrid linear layer)",
                          r["decode_gbs"] * ws, "GB/s", r["decode_ms"], "f32",
                          {"workload": "config 5a: gated DeltaNet, HK16 H48 DK=DV=128, B=1 per GPU (replicas), "
                                       f"{r['prefill_tokens']}-token fused prefill then decode",
                           "l2": f"decode: one token through {DN_LAYERS} layer states (151 MB > 126 MB L2)"},
                          hbm_roof(r["decode_gbs"], "state in+out + token inputs per layer launch"),
                          args.steps * DN_LAYERS, clk.stop())
        line["prefill"] = {"ms": round(r["prefill_ms"], 3), "tokens": r["prefill_tokens"],
                           "form": "chunked WY (64-token chunks) + gated norm",
                           "recurrent_ms": round(r["prefill_recurrent_ms"], 3)}
        return finish(line)
    if args.workload == "roll":
        clk = Clocks(local)
        r = run_roll(torch, ops, args, rank, barrier, max_over_ranks)
        line = _base_line(args, ws, "sink-window decode HBM GB/s (config 4, q8 ring, rope-at-read)",
                          r["gbs"] * ws, "GB/s", r["ms"], "q8",
                          {"workload": f"config 4: H16 KV8 D128, batch {args.roll_batch}, 4 sinks + 4096 ring, "
                                       f"{r['steps']} consecutive decode steps from fill 3076 (crossing "
                                       f"evictions)", "l2": "cache ~150 MB >> L2 only partly"},
                          hbm_roof(r["gbs"], "mean algorithmic bytes per step / mean step time (fused K+V "
                                             "append, attention, LSE merge)"), 3 * r["steps"], clk.stop())
        line["steps"] = r["steps"]
        return finish(line)

    # ---------------- default: config-2 decode headline + variants ----------------
    variants = [v for v in args.variants.split(",") if v]
    modes = [m for m in args.modes.split(",") if m]
    if "q8" in variants and "q8" not in modes:
        modes.append("q8")
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
                cache.append_kv(kd, vd, L - 1)
                ops.attention(qd, cache, L - 1, out=out)
                oh.copy_(out, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                float(oh[0, 0, 0, 0])     # the host reads the step's result
            ms_e2e = max_over_ranks(time_steps(torch, e2e, args.steps, args.warmup, barrier))
            res["e2e"] = {"value": round(ab * ws / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                          "h2d_bytes_per_step": (qh.numel() + kh.numel() + vh.numel()) * 4,
                          "d2h_bytes_per_step": oh.numel() * 4, "ms_per_step": round(ms_e2e, 4),
                          "path": "bitgpu_b200.ops (ctypes -> libbgattn.so C ABI): bg_kv_append_kv + bg_attention"}
        results[mode] = res
        del cache
        torch.cuda.empty_cache()

    short = argparse.Namespace(**vars(args))
    short.steps, short.warmup = max(3, min(args.steps, 20)), 3
    extra = {}
    if "prefill" in variants:
        pf = run_prefill(torch, ops, short, rank, barrier, max_over_ranks)
        tf = pf["flops"] / (pf["ms"] * 1e-3) / 1e12
        extra["prefill"] = {"metric": "prefill-attn TFLOP/s (config 3)", "value": round(tf * ws, 2),
                            "unit": "TFLOP/s", "ms_per_step": round(pf["ms"], 4), "frac": round(tf / bf16_peak, 4),
                            "peak": bf16_peak, "peak_kind": f"{peak_kind} cuBLAS bf16 burst",
                            "flops_per_step_per_gpu": pf["flops"], "kv_write": pf["kv_write"]}
        pf32 = run_prefill(torch, ops, short, rank, barrier, max_over_ranks, mode="f32", q32=True, kv_write=False)
        t32 = pf32["flops"] / (pf32["ms"] * 1e-3) / 1e12
        tf32_pk = tf32_peak(torch)
        extra["prefill_f32kv_3xtf32"] = {
            "metric": "prefill-attn TFLOP/s (config 3 shape, f32 queries over an f32 cache, 3xTF32 on tcgen05)",
            "value": round(t32 * ws, 2), "unit": "TFLOP/s", "ms_per_step": round(pf32["ms"], 4),
            "flops_note": "algorithmic flops (QK^T + PV once); the kernel issues 3 S and 3 PV tf32 products (x3 executed)",
            "tf32_peak": tf32_pk, "frac_of_tf32_peak": round(t32 / tf32_pk["tflops"], 4) if tf32_pk["tflops"] else None}
        pq = run_prefill(torch, ops, short, rank, barrier, max_over_ranks, mode="q8", q32=True, kv_write=False)
        tq = pq["flops"] / (pq["ms"] * 1e-3) / 1e12
        extra["prefill_q8_f32q"] = {"metric": "prefill-attn TFLOP/s (config 3 shape, f32 queries over a q8 cache: "
                                              "the engine's own prefill call)", "value": round(tq * ws, 2),
                                    "unit": "TFLOP/s", "ms_per_step": round(pq["ms"], 4),
                                    "frac": round(tq / bf16_peak, 4), "peak": bf16_peak}
    if "gated" in variants:
        gs = argparse.Namespace(**vars(short))
        gs.steps = max(20, short.steps)
        r = run_gated(torch, ops, gs, ws, rank, barrier, max_over_ranks)
        extra["gated_d256"] = {"metric": "config 5b gated decode GB/s (split-KV over the GPUs)",
                               "value": round(r["gbs"], 1), "unit": "GB/s", "ms_per_step": round(r["ms"], 4),
                               "frac": round(r["gbs"] / ws / hbm, 4), "scaling": "strong",
                               "exchange": r["exchange"]}
        for k in ("nccl_ms", "ms_1gpu", "strong_scaling_efficiency"):
            if k in r:
                extra["gated_d256"][k] = round(r[k], 4)
        if "strong_scaling_efficiency" in r:
            extra_top = {"gated_d256_strong_scaling_efficiency": round(r["strong_scaling_efficiency"], 4)}
        else:
            extra_top = {}
    if "deltanet" in variants:
        r = run_deltanet(torch, ops, short, rank, barrier, max_over_ranks)
        extra["deltanet"] = {"metric": "config 5a DeltaNet decode GB/s (per GPU, replicas)",
                             "value": round(r["decode_gbs"] * ws, 1), "unit": "GB/s",
                             "decode_ms": round(r["decode_ms"], 4), "frac": round(r["decode_gbs"] / hbm, 4),
                             "prefill_4096_ms": round(r["prefill_ms"], 3),
                             "prefill_4096_recurrent_ms": round(r["prefill_recurrent_ms"], 3)}
    if "roll" in variants:
        rs = argparse.Namespace(**vars(short))
        rs.roll_steps = min(args.roll_steps, 1100)
        r = run_roll(torch, ops, rs, rank, barrier, max_over_ranks)
        extra["roll_q8"] = {"metric": "config 4 sink-window decode GB/s", "value": round(r["gbs"] * ws, 1),
                            "unit": "GB/s", "ms_per_step": round(r["ms"], 4), "frac": round(r["gbs"] / hbm, 4),
                            "steps": r["steps"]}

    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    head = results[modes[0]]
    per_launch = head["bytes"] / (head["ms"] * 1e-3) / 1e9
    line = _base_line(args, ws, METRIC, head["gbs"], "GB/s", head["ms"], modes[0],
                      dict(CONFIG, global_batch_per_gpu=nb, kv_mode=modes[0]),
                      hbm_roof(per_launch, "achieved = algorithmic bytes per launch (2*B*L*KV*rowB + 2*B*H*D*4) / "
                                           "mean duration of one bg_attention call, CUDA events on its stream; "
                                           "traffic = ncu dram read+write bytes per sequence (profiles/) x batch",
                               traffic=profiled_traffic(modes[0], nb)),
                      2 * args.steps, head["clocks"])
    line["roofline"]["algorithmic_bytes"] = head["bytes"]
    line["data"] = "synthetic N(0,1), seeded; KV written through the library's own f16/q8 append"
    line["variants"] = {m: {"value": round(r["gbs"], 2), "unit": "GB/s", "ms_per_step": round(r["ms"], 4),
                            "frac": round(r["per_gpu_gbs"] / hbm, 4), "bytes_per_step_per_gpu": r["bytes"]}
                        for m, r in results.items() if m != modes[0]}
    line["variants"].update(extra)
    if "gated" in variants:
        line.update(extra_top)
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
