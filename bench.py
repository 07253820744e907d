"""Benchmark of the GDR hot path on B200 (one JSON line on rank 0).

Default workload (the one the headline metric is quoted on): chunked GDR
prefill, B=4, T=4096, H=16, d_k=d_v=128, chunk 64, bf16 q/k/v, f32 alpha/beta,
f32 state, synthetic inputs with the benchmark distributions (q, k
L2-normalised N(0,1) rows, v ~ N(0,1), beta = sigmoid(N(0,1)),
alpha = exp(-softplus(N(0,1) + 2))). A step is one launch of the
chunked kernel over the whole batch. With --gpus N (one process per GPU,
torchrun) every rank runs its own batch of (sequence, head) units: the path
shards with no data-path collective, so scaling is weak.

Keys beyond the driver contract: `roofline` (dominant kernel, HBM bound at
this arithmetic intensity, with the tensor-core fraction beside it),
`cpu_baseline` (the f64 oracle restating crates/ops/src/delta.rs, timed on
this host's cores), `e2e` (same metric through the host-buffer C-ABI call,
rhz_gdr_scan_chunked_host, with the copies inside the timed region), `decode` (ragged decode
step: 512 sequences x 16 heads from a 1024-slot fp32 pool), `layer` (the
head-sharded full layer of configs[4] at this N, with its NCCL all-gather),
`clocks`.

`--impl reference` times the reference's CPU implementation of the path (the
oracle port, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, T, H, D, CHUNK = 4, 4096, 16, 128, 64
FLOP_PER_TOKEN_HEAD = 6 * D * D + 2 * CHUNK * (3 * D + 2 * D) + (2 / 3) * CHUNK * CHUNK  # 182,955
# Backward products per 64-position chunk of a (sequence, head), in
# multiply-adds: records [K; Q] K^T and W (1,572,864), forward state chain
# V^T (T b)^T, S W^T, Delta^T pL K (2,621,440), adjoint chain dO^T M,
# dS (pL K)^T, dDelta^T W, dO^T gamma Q (3,670,016), per-chunk gradients
# (9,699,328: [K; Q] K^T, dO Delta^T, Delta dS, dO S0, (dM.P) K, (dM.P)^T Q,
# dDelta S0, T^T dDelta, T^T dW, dDelta V^T, dW K^T, dT T^T, T^T E1,
# dKK K twice, dP P^T); the triangular solve is left out.
BWD_FLOP_PER_CHUNK = 2 * (1_572_864 + 2_621_440 + 3_670_016 + 9_699_328)
DEC_N, DEC_SLOTS = 512, 1024
VL_N, VL_SLOTS = 64, 96
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the chunked kernel on this workload, from an ncu capture of that launch.
NCU_TRAFFIC_BYTES = 229_171_200 + 57_360_896


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return PEAKS_FALLBACK, "fallback"


def algorithmic_bytes(b, t, h, d, with_state_in=False):
    tok_heads = b * t * h
    per = 3 * d * 2 + d * 2 + 8  # q, k, v, o (bf16) + alpha, beta (f32)
    states = b * h * d * d * 4 * (2 if with_state_in else 1)
    return tok_heads * per + states


def decode_bytes(n, h, d):
    # state read + write (f32), q/k/v in, o out (bf16), alpha/beta
    return n * h * (2 * d * d * 4 + 3 * d * 2 + 8 + d * 2)


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons, polled through NVML
    every 2 ms while `active` is set: inside the headline timed region and
    every timed sub-measurement (the headline region alone lasts a few ms)."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.active = False
        self._stop = threading.Event()
        self.thread = None
        self.max_mhz = None

    def start(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                try:
                    h = N.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
                except Exception:
                    h = None
            self.h = h if h is not None else N.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self.getreasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self.h = None
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        N = self.N
        while not self._stop.is_set():
            if self.active:
                try:
                    mhz = N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)
                    reasons = self.getreasons(self.h)
                    if self.active:
                        self.samples.append((mhz, reasons))
                except Exception:
                    pass
            time.sleep(0.002)

    def stop(self):
        if self.thread is None:
            return None
        self._stop.set()
        self.thread.join(timeout=2)
        if not self.samples:
            return None
        names = set()
        for _, bits in self.samples:
            for nm, const, default in self.REASONS:
                if bits & getattr(self.N, const, default):
                    names.add(nm)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "sm_min_mhz": min(m for m, _ in self.samples),
                "reasons": sorted(names),
                "source": "NVML, 2 ms polling inside the timed regions"}


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(seed, dev):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    n = torch.nn.functional.normalize
    q = n(torch.randn(B, T, H, D, device=dev, generator=g), dim=-1).to(torch.bfloat16)
    k = n(torch.randn(B, T, H, D, device=dev, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, H, D, device=dev, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=g))
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, device=dev, generator=g) + 2))
    return q, k, v, alpha.contiguous(), beta.contiguous()


def cpu_reference_rate(sample_b: int, min_seconds: float, threads: int):
    """Tokens/s of the f64 oracle (crates/ops/src/delta.rs restated) on
    `sample_b` sequences of the workload, all heads, `threads` host threads."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(1)

    def rows(shape):
        x = rng.standard_normal(shape)
        return x / np.linalg.norm(x, axis=-1, keepdims=True)

    q, k = rows((sample_b, T, H, D)), rows((sample_b, T, H, D))
    v = rng.standard_normal((sample_b, T, H, D))
    beta = 1 / (1 + np.exp(-rng.standard_normal((sample_b, T, H))))
    alpha = np.exp(-np.log1p(np.exp(rng.standard_normal((sample_b, T, H)) + 2)))
    O.lib()
    reps, t0 = 0, time.perf_counter()
    while True:
        O.gdr_dense(q, k, v, alpha, beta, nthreads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds and reps >= 1:
            break
    return reps * sample_b * T / el, reps, el


def prefill_config(world):
    """The headline workload's config, identical in both arms."""
    return {"workload": "chunked GDR prefill B=4 T=4096 H=16 d=128 chunk=64",
            "global_batch": B * world, "seq_len": T, "heads": H, "head_dim": D,
            "chunk": CHUNK, "parallelism": f"shard{world} over (sequence, head)",
            "l2": "inputs larger than L2 (2 x 270 MB sets, alternated)"}


def run_reference(args):
    """--impl reference: the reference's CPU implementation (oracle port)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    sb = 1  # one sequence (4096 tokens x 16 heads) per step: a bounded sample

    def rows(shape):
        x = rng.standard_normal(shape)
        return x / np.linalg.norm(x, axis=-1, keepdims=True)

    q, k = rows((sb, T, H, D)), rows((sb, T, H, D))
    v = rng.standard_normal((sb, T, H, D))
    beta = 1 / (1 + np.exp(-rng.standard_normal((sb, T, H))))
    alpha = np.exp(-np.log1p(np.exp(rng.standard_normal((sb, T, H)) + 2)))
    O.lib()
    for _ in range(args.warmup):
        O.gdr_dense(q, k, v, alpha, beta, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.gdr_dense(q, k, v, alpha, beta, nthreads=threads)
    el = time.perf_counter() - t0
    rate = args.steps * sb * T / el
    sample = f"{sb} of {B} sequences per step ({T} tokens x {H} heads, d={D}), f64"
    line = {
        "impl": "reference", "metric": "GDR prefill tokens/s", "value": rate, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": prefill_config(world),
        "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    from rhizome_b200 import capi, ops

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    capi.lib()
    peaks, peaks_kind = load_peaks()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    # Two input sets (2 x 270 MB > L2), alternated between steps.
    sets = [make_inputs(1000 * rank + s, dev) for s in range(2)]
    o = torch.empty((B, T, H, D), device=dev, dtype=torch.bfloat16)
    fin = torch.empty((B, H, D, D), device=dev, dtype=torch.float32)
    ws_n = int(capi.lib().rhz_gdr_workspace_bytes(B, T, H, D, capi.RHZ_DTYPE_BF16, 0))
    ws = torch.empty(max(ws_n, 1), device=dev, dtype=torch.uint8)

    def launch(i):
        q, k, v, a, b = sets[i % 2]
        capi.call("rhz_gdr_scan_chunked", o.data_ptr(), fin.data_ptr(), q.data_ptr(),
                  k.data_ptr(), v.data_ptr(), a.data_ptr(), b.data_ptr(), None, None, CHUNK, B, T,
                  H, D, capi.RHZ_DTYPE_BF16, ws.data_ptr(), ws_n, sptr)

    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.active = True
    start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        launch(i)
        ev[i][1].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    clocks.active = False
    barrier(world)
    torch.cuda.synchronize()
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)
    kernel_ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    kernel_ms = max_over_ranks(kernel_ms, world)
    tokens = B * T * world * args.steps
    value = tokens / (elapsed_ms / 1e3)

    # Roofline of the dominant kernel (the chunked prefill).
    abytes = algorithmic_bytes(B, T, H, D)
    aflops = FLOP_PER_TOKEN_HEAD * B * T * H
    gbs = abytes / (kernel_ms / 1e3) / 1e9
    tflops = aflops / (kernel_ms / 1e3) / 1e12
    roofline = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                "traffic": args.traffic if args.traffic else NCU_TRAFFIC_BYTES,
                "peaks": f"of {peaks_kind}",
                "kernel": "gdr_chunk_grid_kernel", "kernel_ms": round(kernel_ms, 4),
                "algorithmic_bytes": abytes, "algorithmic_flops": aflops,
                "tensor": {"achieved": round(tflops, 1), "peak": peaks["bf16_tflops"],
                           "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4)}}

    # End to end through the host-buffer C-ABI call (rhz_gdr_scan_chunked_host):
    # pinned host inputs in, host outputs and final states out, every step;
    # the library pipelines the copies against the scan over slabs of
    # positions.
    hq, hk, hv, ha, hb = (x.cpu().pin_memory() for x in sets[0])
    ho = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    hfin = torch.empty(fin.shape, dtype=fin.dtype, pin_memory=True)
    ws_bytes = capi.lib().rhz_gdr_host_workspace_bytes(B, T, H, D, capi.RHZ_DTYPE_BF16, 0)
    hws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    slab = min((T + 63) // 64 * 64, max(256, ((T + 7) // 8 + 63) // 64 * 64))
    n_slabs = (T + slab - 1) // slab
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, ha, hb)) + n_slabs * (3 * B + 1) * 4
    d2h = ho.numel() * ho.element_size() + hfin.numel() * hfin.element_size()

    def e2e_step():
        capi.call("rhz_gdr_scan_chunked_host", ho.data_ptr(), hfin.data_ptr(), hq.data_ptr(),
                  hk.data_ptr(), hv.data_ptr(), ha.data_ptr(), hb.data_ptr(), None, None, CHUNK,
                  B, T, H, D, capi.RHZ_DTYPE_BF16, hws.data_ptr(), ws_bytes, sptr)

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.active = True
    s2.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e2.record(stream)
    torch.cuda.synchronize()
    clocks.active = False
    e2e_ms = max_over_ranks(s2.elapsed_time(e2), world)
    e2e_value = B * T * world * e2e_steps / (e2e_ms / 1e3)

    # Ragged decode step (512 sequences x 16 heads, 1024-slot fp32 pool).
    pool = torch.randn((DEC_SLOTS, H, D, D), device=dev) * 0.02
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    slots = torch.randperm(DEC_SLOTS, device=dev, generator=g)[:DEC_N].to(torch.int32)
    dqk = [sets[0][i][0, :DEC_N].contiguous() for i in range(3)]
    da1, db1 = sets[0][3][0, :DEC_N].contiguous(), sets[0][4][0, :DEC_N].contiguous()
    o1 = torch.empty_like(dqk[0])

    def dec():
        capi.call("rhz_gdr_step", o1.data_ptr(), pool.data_ptr(), slots.data_ptr(),
                  dqk[0].data_ptr(), dqk[1].data_ptr(), dqk[2].data_ptr(), da1.data_ptr(),
                  db1.data_ptr(), DEC_N, DEC_SLOTS, H, D, capi.RHZ_DTYPE_BF16, sptr)

    for _ in range(5):
        dec()
    torch.cuda.synchronize()
    dsteps = 50
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.active = True
    s3.record(stream)
    for _ in range(dsteps):
        dec()
    e3.record(stream)
    torch.cuda.synchronize()
    clocks.active = False
    dec_ms = max_over_ranks(s3.elapsed_time(e3) / dsteps, world)
    dbytes = decode_bytes(DEC_N, H, D)
    dgbs = dbytes / (dec_ms / 1e3) / 1e9
    decode = {"metric": "GDR decode tokens/s", "value": DEC_N * world / (dec_ms / 1e3),
              "unit": "tokens/s", "ms_per_step": round(dec_ms, 4),
              "config": {"sequences": DEC_N, "heads": H, "head_dim": D, "slots": DEC_SLOTS,
                         "dtype": "bf16 q/k/v, f32 state"},
              "roofline": {"bound": "hbm", "achieved": round(dgbs, 1), "peak": peaks["hbm_gbs"],
                           "unit": "GB/s", "frac": round(dgbs / peaks["hbm_gbs"], 4),
                           "kernel": "gdr_step_kernel", "algorithmic_bytes": dbytes}}

    # Input producer (conv + norms + gates) and output norm at the prefill
    # shape: HBM-bound kernels, timed per launch on the device.
    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        sa, sb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.active = True
        sa.record(stream)
        for _ in range(n):
            fn()
        sb.record(stream)
        torch.cuda.synchronize()
        clocks.active = False
        return max_over_ranks(sa.elapsed_time(sb) / n, world)

    xq, xk, xv = sets[0][0], sets[0][1], sets[0][2]
    bl, al = sets[0][3], sets[0][4]
    gp = torch.Generator(device=dev).manual_seed(9 + rank)
    a_head = torch.randn(H, device=dev, generator=gp)
    conv_w = torch.randn((3, H, D, 4), device=dev, generator=gp) * 0.5
    conv_b = torch.randn((3, H, D), device=dev, generator=gp) * 0.1
    conv_state = torch.randn((B, 3, H, D, 3), device=dev, generator=gp)
    pq, pk, pv = torch.empty_like(xq), torch.empty_like(xq), torch.empty_like(xq)
    pa, pb = torch.empty_like(bl), torch.empty_like(bl)
    n_tok = B * T

    def prep():
        capi.call("rhz_gdr_prep", pq.data_ptr(), pk.data_ptr(), pv.data_ptr(), pa.data_ptr(),
                  pb.data_ptr(), xq.data_ptr(), xk.data_ptr(), xv.data_ptr(), bl.data_ptr(),
                  al.data_ptr(), a_head.data_ptr(), conv_w.data_ptr(), conv_b.data_ptr(),
                  conv_state.data_ptr(), None, None, B, T, n_tok, B, H, D, float(D) ** 0.5,
                  capi.RHZ_DTYPE_BF16, 0, sptr)

    prep_ms = timed(prep, 20)
    pbytes = n_tok * H * (6 * D * 2 + 16) + B * 3 * H * D * 3 * 4 * 2
    pgbs = pbytes / (prep_ms / 1e3) / 1e9
    gscale = torch.randn(D, device=dev, generator=gp)
    # The norm runs in place over 4 x the prefill's rows (268 MB, above L2)
    # so that repeated launches do not read from L2.
    n_norm = 4 * n_tok
    gx = torch.randn((n_norm, H, D), device=dev, generator=gp).to(torch.bfloat16)

    def gnorm():
        capi.call("rhz_groupnorm_heads", gx.data_ptr(), gx.data_ptr(), gscale.data_ptr(), n_norm,
                  H, D, 1e-6, capi.RHZ_DTYPE_BF16, sptr)

    gn_ms = timed(gnorm, 20)
    gbytes = n_norm * H * D * 2 * 2
    del gx
    ggbs = gbytes / (gn_ms / 1e3) / 1e9
    producer = {"metric": "GDR input producer tokens/s", "value": n_tok * world / (prep_ms / 1e3),
                "unit": "tokens/s", "ms_per_step": round(prep_ms, 4),
                "config": {"tokens": n_tok, "heads": H, "head_dim": D,
                           "dtype": "bf16 in/out, f32 gates and conv state"},
                "roofline": {"bound": "hbm", "achieved": round(pgbs, 1), "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": round(pgbs / peaks["hbm_gbs"], 4),
                             "kernel": "gdr_prep_tma_kernel", "algorithmic_bytes": pbytes}}
    outnorm = {"metric": "groupnorm_heads tokens/s", "value": n_norm * world / (gn_ms / 1e3),
               "unit": "tokens/s", "ms_per_step": round(gn_ms, 4),
               "config": {"rows": n_norm, "heads": H, "head_dim": D, "dtype": "bf16, in place"},
               "roofline": {"bound": "hbm", "achieved": round(ggbs, 1), "peak": peaks["hbm_gbs"],
                            "unit": "GB/s", "frac": round(ggbs / peaks["hbm_gbs"], 4),
                            "kernel": "groupnorm_heads_kernel", "algorithmic_bytes": gbytes}}

    # Varlen packed prefill: 64 sequences with seeded lengths
    # U{1..8192} in one packed stream, H=16, each from its own N(0, 0.02^2)
    # slot state, final states written back. Timed per launch.
    import numpy as np
    vl = np.random.default_rng(8192 + rank).integers(1, 8193, size=VL_N)
    vcu = torch.tensor(np.concatenate([[0], np.cumsum(vl)]), dtype=torch.int32, device=dev)
    vtok = int(vl.sum())
    gv = torch.Generator(device=dev).manual_seed(31 + rank)
    nrm = torch.nn.functional.normalize
    vq = nrm(torch.randn((vtok, H, D), device=dev, generator=gv), dim=-1).to(torch.bfloat16)
    vk = nrm(torch.randn((vtok, H, D), device=dev, generator=gv), dim=-1).to(torch.bfloat16)
    vv = torch.randn((vtok, H, D), device=dev, generator=gv).to(torch.bfloat16)
    vb = torch.sigmoid(torch.randn((vtok, H), device=dev, generator=gv))
    va = torch.exp(-torch.nn.functional.softplus(torch.randn((vtok, H), device=dev, generator=gv) + 2))
    vpool = torch.randn((VL_SLOTS, H, D, D), device=dev, generator=gv) * 0.02
    vslots = torch.randperm(VL_SLOTS, device=dev, generator=gv)[:VL_N].to(torch.int32)
    vo = torch.empty_like(vq)
    vws_n = int(capi.lib().rhz_gdr_varlen_workspace_bytes(VL_N, H, D, capi.RHZ_DTYPE_BF16))
    vws = torch.empty(max(vws_n, 1), device=dev, dtype=torch.uint8)

    def varlen():
        capi.call("rhz_gdr_varlen_fwd", vo.data_ptr(), vpool.data_ptr(), vslots.data_ptr(),
                  vcu.data_ptr(), vq.data_ptr(), vk.data_ptr(), vv.data_ptr(), va.data_ptr(),
                  vb.data_ptr(), VL_N, vtok, VL_SLOTS, H, D, capi.RHZ_DTYPE_BF16, 0,
                  vws.data_ptr(), vws_n, sptr)

    vl_ms = timed(varlen, 5)
    vbytes = vtok * H * (3 * D * 2 + D * 2 + 8) + VL_N * H * D * D * 4 * 2
    vflops = FLOP_PER_TOKEN_HEAD * vtok * H
    vgbs = vbytes / (vl_ms / 1e3) / 1e9
    vtf = vflops / (vl_ms / 1e3) / 1e12
    varlen_line = {
        "metric": "GDR varlen prefill tokens/s", "value": vtok * world / (vl_ms / 1e3),
        "unit": "tokens/s", "ms_per_step": round(vl_ms, 4),
        "config": {"sequences": VL_N, "tokens": vtok, "lengths": "U{1..8192}, seeded",
                   "heads": H, "head_dim": D, "slots": VL_SLOTS,
                   "kernel_form": "grid (chain and producer CTAs)"},
        "roofline": {"bound": "hbm", "achieved": round(vgbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(vgbs / peaks["hbm_gbs"], 4),
                     "algorithmic_bytes": vbytes, "algorithmic_flops": vflops,
                     "tensor": {"achieved": round(vtf, 1), "peak": peaks["bf16_tflops"],
                                "unit": "TFLOP/s", "frac": round(vtf / peaks["bf16_tflops"], 4)}}}
    del vq, vk, vv, vo

    # Varlen packing (the index/byte work beside the recurrence): slot states
    # gathered into a dense batch (the decode pool's shape), and padded token
    # rows packed by cu_seqlens (the varlen prefill's stream).
    gdense = torch.empty((DEC_N, H, D, D), device=dev)

    def gather():
        capi.call("rhz_varlen_gather_states", gdense.data_ptr(), pool.data_ptr(), slots.data_ptr(),
                  DEC_N, DEC_SLOTS, H, D, sptr)

    ga_ms = timed(gather, 20)
    gabytes = 2 * DEC_N * H * D * D * 4
    row_bytes = H * D * 2
    padded = torch.empty((VL_N, 8192, H, D), device=dev, dtype=torch.bfloat16)
    packed = torch.empty((vtok, H, D), device=dev, dtype=torch.bfloat16)

    def pack():
        capi.call("rhz_varlen_pack_tokens", packed.data_ptr(), padded.data_ptr(), vcu.data_ptr(),
                  VL_N, 8192, row_bytes, sptr)

    pk_ms = timed(pack, 20)
    pkbytes = 2 * vtok * row_bytes
    del padded, packed, gdense
    ga_gbs = gabytes / (ga_ms / 1e3) / 1e9
    pk_gbs = pkbytes / (pk_ms / 1e3) / 1e9
    packing = {
        "gather_states": {"ms": round(ga_ms, 4), "config": f"{DEC_N} x {H} states of {D}x{D} f32 "
                          f"from a {DEC_SLOTS}-slot pool", "algorithmic_bytes": gabytes,
                          "roofline": {"bound": "hbm", "achieved": round(ga_gbs, 1),
                                       "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                       "frac": round(ga_gbs / peaks["hbm_gbs"], 4),
                                       "kernel": "gather_states_kernel"}},
        "pack_tokens": {"ms": round(pk_ms, 4), "config": f"{vtok} rows of {row_bytes} B from "
                        f"[{VL_N}, 8192] padded", "algorithmic_bytes": pkbytes,
                        "roofline": {"bound": "hbm", "achieved": round(pk_gbs, 1),
                                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                     "frac": round(pk_gbs / peaks["hbm_gbs"], 4),
                                     "kernel": "pack_tokens_kernel"}}}

    # Backward of the scan at the prefill shape: the chunked tensor-core form
    # (records, forward and adjoint state chains, per-chunk gradients), with
    # the fp32 reverse scan (state checkpoints every 8 positions) timed
    # beside it for reference.
    dO = torch.randn((B, T, H, D), device=dev, generator=gp).to(torch.bfloat16)
    bws_bytes = int(capi.lib().rhz_gdr_bwd_workspace_bytes(B, T, H, D))
    bws = torch.empty(bws_bytes, device=dev, dtype=torch.uint8)
    gq, gk, gv = torch.empty_like(xq), torch.empty_like(xq), torch.empty_like(xq)
    ga, gb = torch.empty_like(bl), torch.empty_like(bl)
    q0, k0, v0, a0, b0 = sets[0]

    def bwd():
        capi.call("rhz_gdr_scan_chunked_bwd", gq.data_ptr(), gk.data_ptr(), gv.data_ptr(),
                  ga.data_ptr(), gb.data_ptr(), q0.data_ptr(), k0.data_ptr(), v0.data_ptr(),
                  a0.data_ptr(), b0.data_ptr(), None, dO.data_ptr(), None, B, T, H, D,
                  capi.RHZ_DTYPE_BF16, bws.data_ptr(), bws_bytes, sptr)

    bw_ms = timed(bwd, 3)
    prev_form = ops.set_bwd_kernel("scan")
    try:
        scan_ms = timed(bwd, 1)
    finally:
        ops.set_bwd_kernel(prev_form)
    bw_flops = BWD_FLOP_PER_CHUNK * B * H * ((T + CHUNK - 1) // CHUNK)
    bw_tf = bw_flops / (bw_ms / 1e3) / 1e12
    backward = {"metric": "GDR backward tokens/s", "value": B * T * world / (bw_ms / 1e3),
                "unit": "tokens/s", "ms_per_step": round(bw_ms, 4),
                "algorithmic_flops": bw_flops,
                "tensor": {"achieved": round(bw_tf, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                           "frac": round(bw_tf / peaks["bf16_tflops"], 4),
                           "note": "mma.sync fp16 products against the tcgen05 bf16 GEMM peak"},
                "config": {"workload": f"backward of the chunked prefill B={B} T={T} H={H} d={D}",
                           "dtype": "bf16 inputs and gradients; fp16 operands, fp32 accumulation"},
                "kernels": ["gdr_bwdtc_rec_kernel", "gdr_bwdtc_chain_kernel<forward>",
                            "gdr_bwdtc_chain_kernel<adjoint>", "gdr_bwdtc_grad_kernel"],
                "fp32_scan_ms": round(scan_ms, 3)}
    del dO, bws, gq, gk, gv
    # Clock samples from inside the headline timed region and every timed
    # sub-measurement above (the headline region alone lasts a few ms).
    clock_info = clocks.stop()

    # The head-sharded full layer at this N: the NCCL all-gather
    # of per-head outputs is the one collective of the path.
    layer = None if args.no_layer else layer_measure(args, world, rank, local, 3, 1)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        rate, reps, el = cpu_reference_rate(1, 5.0, threads)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"1 of {B} sequences ({T} tokens x {H} heads, d={D}), f64, "
                         f"{reps} repetition(s) in {el:.1f} s"}

    if rank == 0:
        line = {
            "metric": "GDR prefill tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": prefill_config(world),
            "roofline": roofline, "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / e2e_steps, 4),
                    "call": f"rhz_gdr_scan_chunked_host, pinned host buffers, {n_slabs} slabs "
                            f"of {slab} positions pipelined"},
            "gpu_launches": args.steps, "clocks": clock_info, "decode": decode,
            "producer": producer, "output_norm": outnorm, "varlen_prefill": varlen_line,
            "packing": packing, "backward": backward, "layer": layer,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def layer_measure(args, world, rank, local, steps, warmup):
    """The full Local-block layer: B=8, T=32768, H=64, d=128,
    heads split evenly over the ranks, per-head outputs all-gathered (NCCL)
    into [B, T, H*d] on every rank. Total work is fixed (strong scaling).
    Every rank runs the same collectives in the same order; returns the
    measurement dict (meaningful on rank 0)."""
    import torch
    from rhizome_b200.layer import gdr_layer_sharded, gdr_layer_sharded_slabs

    dev = torch.device("cuda", local)
    LB, LT, LH = 8, 32768, 64
    if LH % world:
        raise SystemExit(f"H = {LH} heads do not split over {world} ranks")
    hs = LH // world
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    n = torch.nn.functional.normalize
    q = torch.empty((LB, LT, hs, D), device=dev, dtype=torch.bfloat16)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    for bb in range(LB):  # generate per sequence to bound temporaries
        q[bb] = n(torch.randn(LT, hs, D, device=dev, generator=g), dim=-1).to(torch.bfloat16)
        k[bb] = n(torch.randn(LT, hs, D, device=dev, generator=g), dim=-1).to(torch.bfloat16)
        v[bb] = torch.randn(LT, hs, D, device=dev, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(LB, LT, hs, device=dev, generator=g))
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(LB, LT, hs, device=dev, generator=g) + 2))
    stream = torch.cuda.current_stream(dev)
    ev = []

    def step(record):
        if record:
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev.append((a0, a1))
            a0.record(stream)
            if args.slab:
                out = gdr_layer_sharded_slabs(q, k, v, alpha, beta, slab=args.slab)
                a1.record(stream)  # compute and gathers interleave: no split
            else:
                out = gdr_layer_sharded(q, k, v, alpha, beta,
                                        compute=lambda *x: _timed_compute(x, a1, stream))
        elif args.slab:
            out = gdr_layer_sharded_slabs(q, k, v, alpha, beta, slab=args.slab)
        else:
            out = gdr_layer_sharded(q, k, v, alpha, beta)
        return out

    for _ in range(warmup):
        step(False)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(steps):
        step(True)
    s1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    elapsed = max_over_ranks(s0.elapsed_time(s1), world)
    comp = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / steps, world)
    del q, k, v, alpha, beta
    torch.cuda.empty_cache()
    tokens = LB * LT
    received = (world - 1) * LB * LT * hs * D * 2
    per_step = elapsed / steps
    gather_ms = None if args.slab else max(per_step - comp, 0.0)
    return {
        "metric": "GDR layer tokens/s", "value": tokens * steps / (elapsed / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": per_step, "scaling": "strong",
        "config": {"workload": "full Local-block GDR layer B=8 T=32768 H=64 d=128, heads "
                               "split over ranks, outputs all-gathered (NCCL) into [8, 32768, 8192]"
                               + (f", all-gather overlapped in slabs of {args.slab} positions"
                                  if args.slab else ""),
                   "global_batch": LB, "seq_len": LT, "heads": LH, "head_dim": D,
                   "parallelism": f"heads/{world}"},
        "kernel_only": None if args.slab else {"value": tokens / (comp / 1e3), "unit": "tokens/s",
                                               "ms_per_gpu": round(comp, 4)},
        "allgather": {"bytes_received_per_rank": received,
                      "ms_per_step": None if gather_ms is None else round(gather_ms, 4),
                      "GBps_received_per_rank": (round(received / (gather_ms / 1e3) / 1e9, 1)
                                                 if gather_ms else None),
                      "includes": "NCCL all-gather into rank-major staging + unshard permute",
                      "overlapped_in_slabs": args.slab or None},
    }


def run_layer(args):
    """--workload layer: only the full-layer measurement, as its own line."""
    import torch  # noqa: F401
    from rhizome_b200 import capi

    world, rank, local = dist_setup()
    capi.lib()
    line = layer_measure(args, world, rank, local, args.steps, args.warmup)
    if rank == 0:
        line.update({"higher_is_better": True, "vs_baseline": None, "dtype": "bf16",
                     "data": "synthetic"})
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def _timed_compute(x, ev_done, stream):
    from rhizome_b200 import ops
    out = ops.gdr_scan_chunked(*x)
    ev_done.record(stream)
    return out


def run_case(args):
    """--case NAME: warm-up + --steps launches of one kernel at a size meant
    for an ncu capture (inputs above L2, a few GB at most), timed with CUDA
    events. Not a benchmark line: a fixed launch sequence to profile."""
    import torch
    from rhizome_b200 import capi, ops
    dev = torch.device("cuda", 0)
    capi.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    g = torch.Generator(device=dev).manual_seed(77)
    nrm = torch.nn.functional.normalize

    def qkv(*shape):
        q = nrm(torch.randn(shape, device=dev, generator=g), dim=-1).to(torch.bfloat16)
        k = nrm(torch.randn(shape, device=dev, generator=g), dim=-1).to(torch.bfloat16)
        v = torch.randn(shape, device=dev, generator=g).to(torch.bfloat16)
        b = torch.sigmoid(torch.randn(shape[:-1], device=dev, generator=g))
        a = torch.exp(-torch.nn.functional.softplus(torch.randn(shape[:-1], device=dev, generator=g) + 2))
        return q, k, v, a, b

    if args.case == "decode":  # configs[2]: 512 sequences x 16 heads, 1024-slot pool
        q, k, v, a, b = qkv(DEC_N, H, D)
        pool = torch.randn((DEC_SLOTS, H, D, D), device=dev, generator=g) * 0.02
        slots = torch.randperm(DEC_SLOTS, device=dev, generator=g)[:DEC_N].to(torch.int32)
        o = torch.empty_like(q)

        def fn():
            capi.call("rhz_gdr_step", o.data_ptr(), pool.data_ptr(), slots.data_ptr(), q.data_ptr(),
                      k.data_ptr(), v.data_ptr(), a.data_ptr(), b.data_ptr(), DEC_N, DEC_SLOTS, H, D,
                      capi.RHZ_DTYPE_BF16, sptr)
    elif args.case == "gather":  # 512 x 16 states out of the 1024-slot pool
        pool = torch.randn((DEC_SLOTS, H, D, D), device=dev, generator=g)
        slots = torch.randperm(DEC_SLOTS, device=dev, generator=g)[:DEC_N].to(torch.int32)
        dense = torch.empty((DEC_N, H, D, D), device=dev)

        def fn():
            capi.call("rhz_varlen_gather_states", dense.data_ptr(), pool.data_ptr(),
                      slots.data_ptr(), DEC_N, DEC_SLOTS, H, D, sptr)
    elif args.case == "pack":  # 16 sequences, lengths U{1..8192}, rows of H x d bf16
        import numpy as np
        lens = np.random.default_rng(5).integers(1, 8193, size=16)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
        padded = torch.randn((16, 8192, H, D), device=dev, generator=g).to(torch.bfloat16)
        packed = torch.empty((int(lens.sum()), H, D), device=dev, dtype=torch.bfloat16)

        def fn():
            capi.call("rhz_varlen_pack_tokens", packed.data_ptr(), padded.data_ptr(), cu.data_ptr(),
                      16, 8192, H * D * 2, sptr)
    elif args.case == "norm":  # groupnorm_heads, bf16, in place over 268 MB (4 x the prefill rows)
        x = torch.randn((4 * B * T, H, D), device=dev, generator=g).to(torch.bfloat16)
        scale = torch.randn(D, device=dev, generator=g)

        def fn():
            capi.call("rhz_groupnorm_heads", x.data_ptr(), x.data_ptr(), scale.data_ptr(),
                      4 * B * T, H, D, 1e-6, capi.RHZ_DTYPE_BF16, sptr)
    elif args.case in ("grid", "pair", "solo"):  # the forms of the chunked kernel
        Bc, Tc, Hc = (8, 1024, 64) if args.case == "solo" else (4, 4096, 16)
        q, k, v, a, b = qkv(Bc, Tc, Hc, D)
        ops.set_chunk_kernel(args.case)

        def fn():
            ops.gdr_scan_chunked(q, k, v, a, b)
    elif args.case == "bwd":  # the backward at half the prefill batch (B=2, T=4096, H=16)
        q, k, v, a, b = qkv(2, T, H, D)
        d_o = torch.randn((2, T, H, D), device=dev, generator=g).to(torch.bfloat16)
        ws_n = int(capi.lib().rhz_gdr_bwd_workspace_bytes(2, T, H, D))
        ws = torch.empty(ws_n, device=dev, dtype=torch.uint8)

        def fn():
            ops.gdr_scan_chunked_bwd(q, k, v, a, b, d_o, workspace=ws)
    elif args.case == "varlen":  # configs[3]: the varlen prefill line's packed stream
        import numpy as np
        lens = np.random.default_rng(8192).integers(1, 8193, size=VL_N)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
        ntok = int(lens.sum())
        q, k, v, a, b = qkv(ntok, H, D)
        pool = torch.randn((VL_SLOTS, H, D, D), device=dev, generator=g) * 0.02
        slots = torch.randperm(VL_SLOTS, device=dev, generator=g)[:VL_N].to(torch.int32)
        o = torch.empty_like(q)
        ws_n = int(capi.lib().rhz_gdr_varlen_workspace_bytes(VL_N, H, D, capi.RHZ_DTYPE_BF16))
        ws = torch.empty(max(ws_n, 1), device=dev, dtype=torch.uint8)

        def fn():
            capi.call("rhz_gdr_varlen_fwd", o.data_ptr(), pool.data_ptr(), slots.data_ptr(),
                      cu.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), a.data_ptr(),
                      b.data_ptr(), VL_N, ntok, VL_SLOTS, H, D, capi.RHZ_DTYPE_BF16, 0,
                      ws.data_ptr(), ws_n, sptr)
    else:
        raise SystemExit(f"unknown case {args.case}")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        fn()
    s1.record(stream)
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, "ms_per_launch": s0.elapsed_time(s1) / args.steps}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="prefill", choices=["prefill", "layer"],
                    help="prefill: the headline chunked-prefill batch (weak scaling over "
                         "ranks); layer: the full head-sharded layer with its all-gather")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-layer", action="store_true",
                    help="skip the head-sharded full-layer sub-measurement")
    ap.add_argument("--slab", type=int, default=0,
                    help="--workload layer: overlap the all-gather with compute in slabs of this "
                         "many positions (a multiple of 64; 0 = one call, then one all-gather)")
    ap.add_argument("--case", default=None, choices=["decode", "gather", "pack", "norm", "grid", "pair", "solo", "varlen", "bwd"],
                    help="launch one kernel at a profiling size instead of the benchmark")
    ap.add_argument("--traffic", type=float, default=None,
                    help="measured DRAM bytes per launch of the dominant kernel (ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "layer":
        return run_layer(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
