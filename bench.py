"""Benchmark of the feml mul_mat / mul_mat_id path on B200.

Default workload (N=1 GPU): Q8_0 decode GEMV, weights ne=[K=4096, M=4096]
drawn N(0, 0.02) and quantized to Q8_0, activations [4096, 1] N(0, 1)
quantized on device to Q8_0, seed 1. A step is one mul_mat over one weight
matrix. Other workloads (--config c1|c3|c4|c5) are the remaining shapes of
the hot path, for measurement.

  value  device-timed throughput: CUDA-graph replay of the kernel-level
         entry point on device-resident inputs, rotating through weight
         copies whose total exceeds 2x L2 (every step streams its weights
         from HBM); CUDA events on the launching stream, max over ranks.
  e2e    the same metric through the reference-facing C ABI
         (GraphBuilder -> compile -> write x from pinned host memory ->
         graph_compute -> read y to pinned host memory), every step.

--impl reference times the reference's CPU mul_mat (the C restatement in
oracle/, on all host threads; the Rust reference cannot be built here) on
the same workload; under torchrun only rank 0 runs it.

Multi-GPU (torchrun, --gpus N): by default every rank runs its own replica
of the workload on its own GPU (independent decode streams, weak scaling);
the only collectives are the timing barrier and the max-over-ranks
reduction. --shard rows (c4) / --shard experts (c5) split one workload
across the ranks instead (strong scaling, feml_b200.shard), with the NCCL
all-gather / all-reduce that reassembles the output inside every step.
"""
import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
GEMV_MAX_COLS = 8  # widest activation the decode GEMV takes (gemv.cu kMaxCols)

CONFIGS = {
    "c1": dict(wtype="F32", K=4096, M=4096, N=32, seed=0, dist="uniform", metric="weight-GB/s",
               workload="F32 mul_mat ne=[K=4096,M=4096] x [4096,32], U(-1,1), seed 0"),
    "c2": dict(wtype="Q8_0", K=4096, M=4096, N=1, seed=1, dist="normal", metric="weight-GB/s",
               workload="Q8_0 decode GEMV ne=[K=4096,M=4096], N=1, W~N(0,0.02), x~N(0,1), seed 1"),
    "c3": dict(wtype="Q4_0", K=4096, M=11008, N=512, seed=2, dist="normal", metric="TOPS",
               workload="Q4_0 prefill GEMM ne=[K=4096,M=11008] x [4096,512], seed 2"),
    "c4": dict(wtype="Q4_K", K=14336, M=4096, N=1, seed=3, dist="normal", metric="weight-GB/s",
               workload="Q4_K mul_mat ne=[K=14336,M=4096] x [14336,N], seed 3"),
    "c5": dict(wtype="Q8_0", K=4096, M=14336, N=512, seed=4, dist="normal", metric="weight-GB/s", E=8, n_sel=2,
               workload="Q8_0 mul_mat_id 8 experts ne=[K=4096,M=14336], 512 tokens, top-2, seed 4"),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    except Exception:  # noqa: BLE001
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name):
    """DRAM bytes per launch from a committed ncu summary (a line
    `dram_bytes_per_launch: N` in profiles/<name>.md), or None."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    try:
        with open(p) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1):
        rows = [s for t, s in self.samples if t0 - 0.25 <= t <= t1 + 0.25] or [s for _, s in self.samples]
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [x.strip() for x in r.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ---------------------------------------------------------------------------
def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return ws, rank, local


def reduce_max(v):
    import torch
    import torch.distributed as dist
    if not dist.is_initialized():
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier():
    import torch.distributed as dist
    if dist.is_initialized():
        dist.barrier()


def make_weights(cfg, rank, copies):
    """Synthetic weights on device, quantized by the library's quantizer;
    `copies` distinct buffers holding the same values (L2 rotation)."""
    import torch
    from feml_b200 import DType, ops
    K, M = cfg["K"], cfg["M"]
    E = cfg.get("E", 1)
    g = torch.Generator(device="cuda").manual_seed(cfg["seed"] * 1000 + rank)
    dt = DType[cfg["wtype"]]
    bufs = []
    rb = dt.row_size(K)
    base = torch.empty((E, M, rb if dt != DType.F32 else K * 4), dtype=torch.uint8, device="cuda")
    for e in range(E):
        if cfg["dist"] == "uniform":
            wf = torch.rand((M, K), generator=g, device="cuda") * 2 - 1
        else:
            wf = torch.randn((M, K), generator=g, device="cuda") * 0.02
        if dt == DType.F32:
            base[e] = wf.contiguous().view(torch.uint8).view(M, K * 4)
        else:
            base[e] = ops.quantize(dt, wf.contiguous())
        del wf
    for _ in range(copies):
        bufs.append(base.clone())
    del base
    torch.cuda.synchronize()
    return bufs


def make_x(cfg, rank, N, copies):
    import torch
    g = torch.Generator(device="cuda").manual_seed(cfg["seed"] * 1000 + 500 + rank)
    xs = []
    for _ in range(copies):
        if cfg["dist"] == "uniform":
            xs.append(torch.rand((N, cfg["K"]), generator=g, device="cuda") * 2 - 1)
        else:
            xs.append(torch.randn((N, cfg["K"]), generator=g, device="cuda"))
    return xs


def make_ids(cfg, rank, N):
    rng = np.random.default_rng(cfg["seed"] * 1000 + 900 + rank)
    E, n_sel = cfg["E"], cfg["n_sel"]
    return np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)


def step_units(cfg, N):
    """(bytes streamed per step as the metric counts them, algorithmic bytes
    per step, ops per step)."""
    from feml_b200 import DType
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    wbytes = dt.row_size(K) * M * cfg.get("E", 1)
    n_cols = N * cfg.get("n_sel", 1)
    alg = wbytes + 4 * K * N + 4 * M * n_cols + (4 * n_cols if "E" in cfg else 0)
    ops_ = 2.0 * K * M * n_cols
    return wbytes, alg, ops_


def metric_value(cfg, N, seconds_per_step):
    wbytes, _, ops_ = step_units(cfg, N)
    if cfg["metric"] == "TOPS":
        return ops_ / seconds_per_step / 1e12, "TOPS"
    return wbytes / seconds_per_step / 1e9, "GB/s"


def kernels_per_step(cfg, N):
    from feml_b200 import DType
    dt = DType[cfg["wtype"]]
    if "E" in cfg:
        return 3 if dt != DType.F32 else 2
    if dt == DType.F32:
        return 1
    from feml_b200 import ops
    if ops.mul_mat_workspace(dt, cfg["K"], cfg["M"], N) == 0:
        return 1  # fused GEMV
    tc = dt in (DType.Q8_0, DType.Q4_0) and cfg["K"] % 256 == 0 and N > GEMV_MAX_COLS
    split = (not tc and N > GEMV_MAX_COLS and cfg["K"] % 256 == 0 and
             ops.mul_mat_workspace(dt, cfg["K"], cfg["M"], N) > _planar_bytes(cfg["K"], N))
    return 3 if split else 2  # activation quantizer + GEMM (+ split-K reduction)


def _planar_bytes(K, N):
    """Planar Q8_0 activation bytes (qs, d, sum, each padded to 256 B)."""
    pad = lambda v: (v + 255) // 256 * 256  # noqa: E731
    return pad(N * K) + 2 * pad(N * (K // 32) * 4)


def dominant_kernel(cfg, N):
    from feml_b200 import DType
    dt = DType[cfg["wtype"]]
    tc = dt in (DType.Q8_0, DType.Q4_0) and cfg["K"] % 256 == 0
    if "E" in cfg:
        return "gemm_tc_kernel (grouped, tcgen05)" if tc else "gemm_q_kernel (grouped)"
    if dt == DType.F32:
        return "gemm_f32_pipe_kernel" if cfg["K"] % 4 == 0 else "gemm_f32_exact_kernel"
    if N <= GEMV_MAX_COLS:
        if dt == DType.Q4_K and 12288 <= cfg["K"] <= 16384:
            return "gemv_ks_kernel" if N == 1 else "gemv_ks_cols_kernel"
        return "gemv_kernel"
    return "gemm_tc_kernel (tcgen05)" if tc else "gemm_q_kernel"


# ---------------------------------------------------------------------------
def run_b200(args, cfg, N):
    import torch
    from feml_b200 import DType, ops
    import feml_b200 as F

    ws, rank, local = dist_setup()
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    wbytes, alg_bytes, ops_step = step_units(cfg, N)
    copies = max(1, math.ceil(2.5 * L2_BYTES / wbytes))
    wts = make_weights(cfg, rank, copies)
    xs = make_x(cfg, rank, N, min(copies, 4))
    is_moe = "E" in cfg
    stream = torch.cuda.current_stream()
    if is_moe:
        ids_np = make_ids(cfg, rank, N)
        ids = torch.from_numpy(ids_np).cuda()
        n_sel = cfg["n_sel"]
        outs = [torch.empty((N, n_sel, M), dtype=torch.float32, device="cuda") for _ in range(2)]
        wsz = ops.mul_mat_id_workspace(dt, K, M, N, n_sel, cfg["E"])
        work = torch.empty(max(wsz, 1), dtype=torch.uint8, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")

        def step(i):
            ops.mul_mat_id(dt, wts[i % copies], xs[i % len(xs)], ids, K, out=outs[i % 2], workspace=work,
                           status=status)
    else:
        outs = [torch.empty((N, M), dtype=torch.float32, device="cuda") for _ in range(2)]
        wsz = ops.mul_mat_workspace(dt, K, M, N)
        work = torch.empty(max(wsz, 1), dtype=torch.uint8, device="cuda") if wsz else None
        wview = [w[0] if dt != DType.F32 else w[0].view(torch.float32) for w in wts]

        def step(i):
            ops.mul_mat(dt, wview[i % copies], xs[i % len(xs)], K, out=outs[i % 2], workspace=work)

    # capture the step sequence in CUDA graphs (launch cost off the timeline)
    chunk = min(args.steps, max(copies, 64) if args.steps >= 64 else args.steps)
    chunk = max(1, min(chunk, 1024))
    for i in range(3):
        step(i)
    torch.cuda.synchronize()

    def capture(n):
        if n == 0:
            return None
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for i in range(n):
                step(i)
        return gr

    g_main = capture(chunk)
    g_tail = capture(args.steps % chunk)
    torch.cuda.synchronize()

    def run_steps(k):
        for _ in range(k // chunk):
            g_main.replay()
        if k % chunk:
            if k == args.steps and g_tail is not None:
                g_tail.replay()
            else:
                for i in range(k % chunk):
                    step(i)

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    run_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    barrier()
    ms = e0.elapsed_time(e1)
    ms_max = reduce_max(ms)
    time.sleep(0.25)
    sampler.stop()
    clocks = sampler.summary(t0, t1)

    sec_step = ms_max / 1e3 / args.steps
    per_gpu_val, unit = metric_value(cfg, N, sec_step)
    value = per_gpu_val * ws

    # ---- e2e through the reference-facing C ABI -------------------------------
    e2e = run_e2e(args, cfg, N, dt, wts, copies, ids_np if is_moe else None, local)

    # ---- roofline of the dominant kernel ------------------------------------
    peaks = load_peaks()
    if cfg["metric"] == "TOPS":
        achieved = ops_step / sec_step / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "peak_note": f"bf16 dense {peaks['source']} (the kernel issues f16 tcgen05 MMAs on exact integer / split operands)"}
    else:
        achieved = alg_bytes / sec_step / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_note": f"HBM copy bandwidth, {peaks['source']}"}
    prof_name = f"{args.config}_{cfg['wtype'].lower()}_n{N}"
    tr = profile_traffic(prof_name)
    roof["traffic"] = tr
    roof["kernel"] = dominant_kernel(cfg, N)
    roof["algorithmic_bytes_per_launch"] = alg_bytes
    roof["timing"] = "per-step device time (CUDA events over the graph-replayed steps), includes launch gaps"

    result = {
        "metric": f"mul_mat {'prefill GEMM TOPS' if cfg['metric'] == 'TOPS' else 'decode weight-GB/s'} "
                  f"({args.config}: {cfg['workload']})",
        "value": value, "unit": unit, "n_gpus": ws, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 dot / f32 scale" if dt != DType.F32 else "f32",
        "data": "synthetic (seeded torch.randn weights quantized on device; seeded activations)",
        "config": {"workload": cfg["workload"], "config": args.config, "K": K, "M": M, "N": N,
                   "weights_dtype": cfg["wtype"], "experts": cfg.get("E"), "n_selected": cfg.get("n_sel"),
                   "l2": f"{copies} rotating weight copies ({copies * wbytes / 2**20:.0f} MiB, > 2x L2)",
                   "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU"},
        "roofline": roof,
        "e2e": e2e,
        "gpu_launches": args.steps * kernels_per_step(cfg, N),
        "clocks": clocks,
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg, N, wts[0], budget_s=args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)
    # release graphs before the process group goes away
    del g_main, g_tail
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, cfg, N, dt, wts, copies, ids_np, local):
    """Same metric through the C ABI with host buffers: per step, x from
    pinned host memory -> device (write), graph_compute, y -> pinned host
    memory (read, which synchronizes the stream)."""
    import torch
    import feml_b200 as F
    from feml_b200 import DType, GraphBuilder

    K, M = cfg["K"], cfg["M"]
    be = F.B200Backend.open(local)
    n_plans = min(copies, 24)
    is_moe = ids_np is not None
    w_host = wts[0].cpu().numpy()  # the quantized bytes, uploaded once per plan (outside the timed region)
    plans = []
    for p in range(n_plans):
        g = GraphBuilder()
        if is_moe:
            E, n_sel = cfg["E"], cfg["n_sel"]
            w = g.weight("w", dt, [K, M, E])
            xi = g.input("x", DType.F32, [K, N])
            ii = g.input("ids", DType.I32, [n_sel, N])
            o = g.mul_mat_id(w, xi, ii, n_sel)
        else:
            w = g.weight("w", dt, [K, M])
            xi = g.input("x", DType.F32, [K, N])
            o = g.mul_mat(w, xi)
            ii = None
        g.mark_output(o)
        plan = g.compile(be)
        plan.write_tensor(be, w, w_host)
        if is_moe:
            plan.write_tensor(be, ii, ids_np)
        plans.append((plan, plan.find(xi), plan.find(o), g))
    x_host = torch.randn((N, K), dtype=torch.float32).pin_memory()
    y_elems = N * M * (cfg["n_sel"] if is_moe else 1)
    y_host = torch.empty(y_elems, dtype=torch.float32).pin_memory()
    steps = min(args.steps, args.e2e_steps)
    x_bytes, y_bytes = N * K * 4, y_elems * 4

    def one(i):
        plan, px, po, _ = plans[i % n_plans]
        be.write_ptr(plan.buffers[px.buffer].handle, px.offset, x_host.data_ptr(), x_bytes)
        be.graph_compute(plan)
        be.read_ptr(plan.buffers[po.buffer].handle, po.offset, y_host.data_ptr(), y_bytes)

    for i in range(max(3, min(args.warmup, 50))):
        one(i)
    be.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(steps):
        one(i)
    be.synchronize()
    dt_s = reduce_max(time.perf_counter() - t0)
    v, unit = metric_value(cfg, N, dt_s / steps)
    import torch.distributed as dist
    ws = dist.get_world_size() if dist.is_initialized() else 1
    for plan, *_ in plans:
        plan.release(be)
    be.close()
    return {"value": v * ws, "unit": unit, "h2d_bytes_per_step": x_bytes, "d2h_bytes_per_step": y_bytes,
            "steps": steps, "ms_per_step": dt_s / steps * 1e3,
            "path": "GraphBuilder->compile->write(pinned x)->graph_compute->read(pinned y), libfeml_b200 C ABI"}


# ---------------------------------------------------------------------------
def run_sharded(args, cfg, N):
    """Strong scaling of one workload split across the ranks: --shard rows
    (weight rows, all-gather of the output slices) or --shard experts
    (experts e % world, sum all-reduce of the slot outputs). A step is the
    local kernels plus the collective that leaves the full output on every
    rank; the step sequence (NCCL calls included) is replayed as a CUDA graph."""
    import torch
    import torch.distributed as dist
    from feml_b200 import DType, ops
    from feml_b200.shard import ExpertShardedMulMatId, RowShardedMulMat, local_experts, row_range

    ws, rank, local = dist_setup()
    if ws == 1 and not dist.is_initialized():
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + (os.getpid() % 1000)))
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    wbytes_total, alg_total, ops_total = step_units(cfg, N)
    rb = dt.row_size(K)
    g = torch.Generator(device="cuda").manual_seed(cfg["seed"] * 1000)
    is_moe = args.shard == "experts"
    if is_moe:
        E, n_sel = cfg["E"], cfg["n_sel"]
        n_loc = local_experts(E, rank, ws)
        local_w = torch.empty((max(n_loc, 1), M, rb), dtype=torch.uint8, device="cuda")
        for e in range(E):  # every rank draws all experts from one seed and keeps its own
            wf = torch.randn((M, K), generator=g, device="cuda") * 0.02
            if e % ws == rank:
                local_w[e // ws] = ops.quantize(dt, wf)
            del wf
        local_w = local_w[:n_loc]
        local_bytes = n_loc * M * rb
    else:
        lo, hi, R = row_range(M, rank, ws)
        wf = torch.randn((M, K), generator=g, device="cuda") * 0.02
        local_w = ops.quantize(dt, wf[lo:hi].contiguous())
        del wf
        local_bytes = (hi - lo) * rb
    copies = max(1, math.ceil(2.5 * L2_BYTES / max(local_bytes, 1)))
    wts = [local_w.clone() for _ in range(copies)]
    gx = torch.Generator(device="cuda").manual_seed(cfg["seed"] * 1000 + 500)
    x = torch.randn((N, K), generator=gx, device="cuda")
    if is_moe:
        ids_np = make_ids(cfg, 0, N)
        ids = torch.from_numpy(ids_np).cuda()
        if args.fused:  # one peer-buffer set; the weight copies rotate under it
            mod = ExpertShardedMulMatId(dt, wts[0], K, E, local=True, fused=True, max_tokens=N,
                                        max_selected=n_sel)

            def step(i):
                mod.w_local = wts[i % copies]
                return mod(x, ids)
        else:
            mods = [ExpertShardedMulMatId(dt, w, K, E, local=True) for w in wts]

            def step(i):
                return mods[i % copies](x, ids)
    else:
        if args.fused:  # one peer-buffer set; the weight copies rotate under it
            mod = RowShardedMulMat(dt, wts[0], K, M, local=True, fused=True)

            def step(i):
                mod.w_local = wts[i % copies]
                return mod(x)
        else:
            mods = [RowShardedMulMat(dt, w, K, M, local=True) for w in wts]

            def step(i):
                return mods[i % copies](x)

    chunk = max(1, min(args.steps, max(copies, 16), 256))
    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(chunk):
            step(i)
    torch.cuda.synchronize()
    reps = max(1, args.steps // chunk)
    steps = reps * chunk
    for _ in range(max(1, max(args.warmup, 3) // chunk + 1)):
        gr.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    for _ in range(reps):
        gr.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    barrier()
    ms_max = reduce_max(e0.elapsed_time(e1))
    time.sleep(0.25)
    sampler.stop()
    sec_step = ms_max / 1e3 / steps
    value, unit = metric_value(cfg, N, sec_step)  # the whole job's work per step
    # e2e: x from pinned host memory, the sharded op, y to pinned host memory
    x_host = torch.randn((N, K), dtype=torch.float32).pin_memory()
    y_elems = N * M * (cfg["n_sel"] if is_moe else 1)
    y_host = torch.empty(y_elems, dtype=torch.float32).pin_memory()
    e2e_steps = min(steps, args.e2e_steps)
    for i in range(5):
        x.copy_(x_host, non_blocking=True)
        y_host.copy_(step(i).reshape(-1), non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    tt = time.perf_counter()
    for i in range(e2e_steps):
        x.copy_(x_host, non_blocking=True)
        y_host.copy_(step(i).reshape(-1), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_s = reduce_max(time.perf_counter() - tt) / e2e_steps
    e2e_v, _ = metric_value(cfg, N, e2e_s)
    peaks = load_peaks()
    # ours per step: route + quantize + grouped GEMM (MoE) or GEMV (+ quantize), plus the wait kernel when fused
    n_k = (3 if is_moe else 1 + (1 if ops.mul_mat_workspace(dt, K, M, N) else 0)) + (1 if args.fused else 0)
    result = {
        "metric": f"mul_mat {'mul_mat_id expert-sharded' if is_moe else 'row-sharded'} weight-GB/s "
                  f"({args.config}: {cfg['workload']})",
        "value": value, "unit": unit, "n_gpus": ws, "steps": steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 dot / f32 scale", "data": "synthetic (seeded torch.randn weights quantized on device)",
        "config": {"workload": cfg["workload"], "config": args.config, "K": K, "M": M, "N": N,
                   "weights_dtype": cfg["wtype"], "experts": cfg.get("E"), "n_selected": cfg.get("n_sel"),
                   "parallelism": f"{'expert' if is_moe else 'row'}-sharded x{ws} + " + (
                       "peer-memory stores (fused)" if args.fused else
                       ("NCCL all_reduce" if is_moe else "NCCL all_gather")),
                   "l2": f"{copies} rotating local weight copies ({copies * local_bytes / 2**20:.0f} MiB per rank)"},
        "roofline": {"bound": "hbm", "achieved": alg_total / sec_step / 1e9, "peak": peaks["hbm_gbs"] * ws,
                     "unit": "GB/s", "frac": alg_total / sec_step / 1e9 / (peaks["hbm_gbs"] * ws), "traffic": None,
                     "peak_note": f"{ws} x HBM copy bandwidth ({peaks['source']}); step includes the collective"},
        "e2e": {"value": e2e_v, "unit": unit, "h2d_bytes_per_step": N * K * 4, "d2h_bytes_per_step": y_elems * 4,
                "steps": e2e_steps, "path": "feml_b200.shard wrapper, pinned host x -> device -> pinned host y"},
        "gpu_launches": steps * n_k,
        "clocks": sampler.summary(t0, t1),
    }
    if rank == 0:
        print(json.dumps(result), flush=True)
    del gr
    dist.barrier()
    dist.destroy_process_group()


# ---------------------------------------------------------------------------
def cpu_baseline(cfg, N, wq_dev, budget_s=10.0, threads=None):
    """The reference's CPU mul_mat (oracle/, the C restatement of
    feml-cpu/src/ops/mul_mat.rs:36-57) on a bounded sample of the workload.
    The reference has no quantized kernel: its path is the F32 mul_mat on the
    dequantized weights (dequantized once, as a user of the reference would
    store them) and, as on the device, Q8_0-rounded activations."""
    from oracle import oracle as O
    from feml_b200 import DType
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    threads = threads or (os.cpu_count() or 1)
    wq = wq_dev[0].cpu().numpy() if wq_dev.dim() == 3 else wq_dev.cpu().numpy()
    rng = np.random.default_rng(cfg["seed"])
    x = rng.standard_normal((N, K)).astype(np.float32)
    # sample: enough weight rows that one sample step costs ~0.1-0.5 s
    macs_target = 2e8
    n_cols = N * cfg.get("n_sel", 1)
    rows = int(min(M, max(64, macs_target // (K * n_cols))))
    code = {DType.F32: O.DT_F32, DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K}[dt]
    if dt == DType.F32:
        wf = wq[:rows].view(np.float32).reshape(rows, K)
    else:
        wf = O.dequantize(code, wq[:rows], K)
    xs = x if "E" not in cfg else np.repeat(x, cfg["n_sel"], axis=0)
    t_end = time.perf_counter() + budget_s
    n_iter, t_total = 0, 0.0
    while True:
        t0 = time.perf_counter()
        xf = O.dequantize(O.DT_Q8_0, O.quantize(O.DT_Q8_0, xs), K) if dt != DType.F32 else xs
        O.mul_mat_f32(wf, xf, nthreads=threads)
        t_total += time.perf_counter() - t0
        n_iter += 1
        if time.perf_counter() > t_end or n_iter >= 1000:
            break
    frac = rows / M
    sec_full_step = t_total / n_iter / frac
    v, unit = metric_value(cfg, N, sec_full_step)
    return {"value": v, "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{rows}/{M} weight rows x {n_cols} columns per iteration, {n_iter} iterations "
                      f"({t_total:.1f} s); value scaled to the full step",
            "sec_per_full_step": sec_full_step}


def run_reference(args, cfg, N):
    """The reference's CPU mul_mat on all host threads (the oracle port: the
    Rust reference cannot be built in this image). Each step is a bounded
    sample of the workload (a slice of weight rows, all columns), sized so
    the whole run stays within about a minute; the value is scaled to the
    full step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    from feml_b200 import DType
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    code = {DType.F32: O.DT_F32, DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K}[dt]
    n_cols = N * cfg.get("n_sel", 1)
    total_steps = args.steps + max(args.warmup, 3)
    macs = min(2e8, max(2e5, 60.0 * 1e9 / total_steps))
    rows = int(min(M, max(1, macs // (K * n_cols))))
    threads = max(1, min(os.cpu_count() or 1, rows // 16))
    rng = np.random.default_rng(cfg["seed"])
    if cfg["dist"] == "uniform":
        wf = rng.uniform(-1, 1, (rows, K)).astype(np.float32)
    else:
        wf = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
    wdeq = O.dequantize(code, O.quantize(code, wf), K) if dt != DType.F32 else wf
    x = np.random.default_rng(cfg["seed"] + 1).standard_normal((n_cols, K)).astype(np.float32)

    def sample():
        xf = O.dequantize(O.DT_Q8_0, O.quantize(O.DT_Q8_0, x), K) if dt != DType.F32 else x
        O.mul_mat_f32(wdeq, xf, nthreads=threads)

    for _ in range(max(args.warmup, 3)):
        sample()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sample()
    dt_s = time.perf_counter() - t0
    sec_full = dt_s / args.steps / (rows / M)
    v, unit = metric_value(cfg, N, sec_full)
    print(json.dumps({
        "impl": "reference",
        "metric": f"mul_mat {'prefill GEMM TOPS' if cfg['metric'] == 'TOPS' else 'decode weight-GB/s'} "
                  f"({args.config}: {cfg['workload']})",
        "value": v, "unit": unit, "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": sec_full * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded numpy)",
        "config": {"workload": cfg["workload"], "config": args.config, "K": K, "M": M, "N": N},
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"{rows}/{M} weight rows x {n_cols} columns per step, scaled to the full "
                                   f"step; F32 mul_mat (feml-cpu/src/ops/mul_mat.rs:36-57 restated in C) on "
                                   f"dequantized weights and Q8_0-rounded activations"},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200000)
    ap.add_argument("--warmup", type=int, default=2000)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--tokens", type=int, default=None, help="activation columns N (c4: 1, 8 or 64)")
    ap.add_argument("--e2e-steps", type=int, default=5000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", default="none", choices=["none", "rows", "experts"],
                    help="strong-scaling split of one workload across the ranks (c4: rows, c5: experts)")
    ap.add_argument("--fused", action="store_true",
                    help="peer-memory stores + flags instead of the NCCL collective (--shard rows at decode "
                         "shapes, --shard experts)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    N = args.tokens if args.tokens is not None else cfg["N"]
    if args.impl == "reference":
        run_reference(args, cfg, N)
        return
    if args.shard != "none":
        if (args.shard == "experts") != ("E" in cfg) or cfg["wtype"] == "F32":
            ap.error("--shard rows needs a quantized mul_mat config (c2, c3, c4); --shard experts needs c5")
        run_sharded(args, cfg, N)
        return
    run_b200(args, cfg, N)


if __name__ == "__main__":
    main()
