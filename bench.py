"""Benchmark of the feml mul_mat / mul_mat_id path on B200.

Headline workload (the same at every GPU count, so the driver's per-N values
form a strong-scaling curve): C5, the Q8_0 mul_mat_id MoE layer -- 8 experts
ne=[K=4096, M=14336] drawn N(0, 0.02) and quantized to Q8_0, 512 tokens of
N(0, 1) activations, top-2 expert ids per token drawn uniformly without
replacement. A step is one mul_mat_id over the whole layer.

  N = 1    the unsharded mul_mat_id (route + activation quantization +
           grouped tcgen05 GEMM on one GPU).
  N > 1    expert-sharded across the ranks (expert e on rank e % N), the
           combine inside every step: by default each slot goes to the rank
           that owns its token (token t on rank t // ceil(512 / N)) by peer
           stores from the GEMM epilogue plus a bounded flag wait
           (--combine owner); --combine replicate stores every slot on every
           rank, --combine nccl all-reduces the slot tensor.

  value  device-timed throughput (weight bytes per second, whole job):
         CUDA-graph replay of the steps on device-resident inputs, CUDA
         events on the launching stream after a barrier and a synchronize,
         max over ranks.
  e2e    the same metric through the public API with host buffers: at N=1
         the reference-facing C ABI (GraphBuilder -> compile -> write x and
         ids from pinned host memory -> graph_compute -> read y to pinned
         host memory); at N>1 the feml_b200.shard wrapper (x and ids copied
         in, each rank's own tokens' slots copied out).
  extras the other shapes of the path on the same GPUs: at N=1 the decode
         GEMV (C2, Q8_0 4096x4096, N=1, with its own e2e), the prefill GEMM
         (C3, Q4_0 11008x4096x512, TOPS), C4 (Q4_K 4096x14336 at N=1/8/64)
         and C1 (F32); at N>1 the row-sharded C4 decode step and the other
         two C5 combines.

Inputs of both arms come from the same seeded numpy draws: weights of
expert e in 512-row chunks from default_rng([seed, e, chunk]), activations
from default_rng([seed, 1000]), ids from default_rng([seed, 2000]); the
quantized weight bytes are the device quantizer's (bit-identical to the
oracle's).

--impl reference times the reference's CPU mul_mat (the C restatement in
oracle/ of feml-cpu/src/ops/mul_mat.rs:36-57, on all host threads; the Rust
reference cannot be built in this image) on a bounded row sample of the
same workload; under torchrun only rank 0 runs it. It imports nothing from
feml_b200.
"""
import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
CHUNK_ROWS = 512  # weight rows per seeded draw

# ggml block size and bytes per block (feml-core/src/dtype.rs:52-72)
BLOCK = {"F32": (1, 4), "Q8_0": (32, 34), "Q4_0": (32, 18), "Q4_K": (256, 144)}
DT_CODE = {"F32": 5, "Q4_0": 7, "Q8_0": 11, "Q4_K": 15}  # dtype.rs:14-35 discriminants

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


def row_size(wtype, K):
    bs, ts = BLOCK[wtype]
    return K // bs * ts


def step_units(cfg, N):
    """(weight bytes per step, algorithmic bytes W + x + y (+ ids), ops 2*M*K per output column)."""
    K, M = cfg["K"], cfg["M"]
    wbytes = row_size(cfg["wtype"], K) * M * cfg.get("E", 1)
    n_cols = N * cfg.get("n_sel", 1)
    alg = wbytes + 4 * K * N + 4 * M * n_cols + (4 * n_cols if "E" in cfg else 0)
    return wbytes, alg, 2.0 * K * M * n_cols


def metric_value(cfg, N, seconds_per_step):
    wbytes, _, ops_ = step_units(cfg, N)
    if cfg["metric"] == "TOPS":
        return ops_ / seconds_per_step / 1e12, "TOPS"
    return wbytes / seconds_per_step / 1e9, "GB/s"


def metric_name(cfg_name, cfg):
    kind = "prefill GEMM TOPS" if cfg["metric"] == "TOPS" else (
        "mul_mat_id weight-GB/s" if "E" in cfg else "decode weight-GB/s")
    return f"mul_mat {kind} ({cfg_name}: {cfg['workload']})"


def config_dict(cfg_name, cfg, N, world):
    """The config both arms print (identical by construction)."""
    if "E" in cfg:
        par = "single GPU" if world == 1 else f"expert-sharded x{world}"
    else:
        par = "single GPU" if world == 1 else f"row-sharded x{world}"
    return {"workload": cfg["workload"], "config": cfg_name, "K": cfg["K"], "M": cfg["M"], "N": N,
            "weights_dtype": cfg["wtype"], "experts": cfg.get("E"), "n_selected": cfg.get("n_sel"),
            "seed": cfg["seed"], "parallelism": par}


# ---------------------------------------------------------------------------
# Seeded inputs, shared by both arms
# ---------------------------------------------------------------------------
def host_weight_rows(cfg, expert, r0, r1, threads=None):
    """f32 rows [r0, r1) of expert `expert`'s weight (ggml ne=[K, M] rows)."""
    K = cfg["K"]
    out = np.empty((r1 - r0, K), np.float32)

    def fill(c):
        a, b = c * CHUNK_ROWS, min(cfg["M"], (c + 1) * CHUNK_ROWS)
        lo, hi = max(a, r0), min(b, r1)
        if lo >= hi:
            return
        rng = np.random.default_rng([cfg["seed"], expert, c])
        if cfg["dist"] == "uniform":
            blk = rng.random((hi - a, K), dtype=np.float32) * np.float32(2) - np.float32(1)
        else:
            blk = rng.standard_normal((hi - a, K), dtype=np.float32) * np.float32(0.02)
        out[lo - r0:hi - r0] = blk[lo - a:]

    chunks = range(r0 // CHUNK_ROWS, (r1 + CHUNK_ROWS - 1) // CHUNK_ROWS)
    with ThreadPoolExecutor(threads or min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, chunks))
    return out


def host_x(cfg, N):
    rng = np.random.default_rng([cfg["seed"], 1000])
    if cfg["dist"] == "uniform":
        return rng.random((N, cfg["K"]), dtype=np.float32) * np.float32(2) - np.float32(1)
    return rng.standard_normal((N, cfg["K"]), dtype=np.float32)


def host_ids(cfg, N):
    rng = np.random.default_rng([cfg["seed"], 2000])
    return np.stack([rng.permutation(cfg["E"])[:cfg["n_sel"]] for _ in range(N)]).astype(np.int32)


_WEIGHTS = {}


def device_weights(cfg, experts, rows=None):
    """Quantized weights of the listed experts on the current device, uint8
    [len(experts), M, row_bytes] (F32: the f32 bytes), quantized by the
    library's quantizer expert by expert (kept for the next caller)."""
    import torch
    from feml_b200 import DType, ops
    K, M = cfg["K"], cfg["M"]
    r0, r1 = rows if rows else (0, M)
    key = (cfg["workload"], tuple(experts), r0, r1)
    if key in _WEIGHTS:
        return _WEIGHTS[key]
    rb = row_size(cfg["wtype"], K)
    out = torch.empty((len(experts), r1 - r0, rb), dtype=torch.uint8, device="cuda")
    for j, e in enumerate(experts):
        wf = torch.from_numpy(host_weight_rows(cfg, e, r0, r1)).cuda()
        if cfg["wtype"] == "F32":
            out[j] = wf.view(torch.uint8).view(r1 - r0, rb)
        else:
            out[j] = ops.quantize(DType[cfg["wtype"]], wf)
        del wf
    torch.cuda.synchronize()
    _WEIGHTS.clear()  # keep only the latest set
    _WEIGHTS[key] = out
    return out


# ---------------------------------------------------------------------------
# Plumbing: ranks, clocks, timing
# ---------------------------------------------------------------------------
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

    def summary(self, windows):
        rows = [s for t, s in self.samples if any(a - 0.25 <= t <= b + 0.25 for a, b in windows)]
        rows = rows or [s for _, s in self.samples]
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


def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
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


class Timer:
    """Device time of `steps` calls of step(i), replayed as CUDA graphs.

    Three eager steps first (one-time setup stays out of the capture), then
    the steps are captured in graphs of `chunk` steps (plus a tail graph);
    warm-up replays every graph at least once and at least `warmup` steps;
    the timed region is one replay of the whole sequence, between CUDA
    events on the launching stream, with a barrier and a synchronize on both
    sides; the result is the max over ranks."""

    def __init__(self, windows):
        self.windows = windows  # wall-clock spans of timed regions (clock sampling)
        self.graphs = []

    def run(self, step, steps, warmup, chunk_hint=64):
        import torch
        chunk = max(1, min(steps, max(chunk_hint, 16), 512))
        n_full, tail = divmod(steps, chunk)
        for i in range(min(3, steps)):
            step(i)
        torch.cuda.synchronize()

        def capture(n):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(n):
                    step(i)
            return g

        g_main = capture(chunk) if n_full else None
        g_tail = capture(tail) if tail else None
        self.graphs += [g for g in (g_main, g_tail) if g is not None]
        torch.cuda.synchronize()
        done = 0
        while True:  # warm-up: each graph at least once, at least `warmup` steps
            if g_main is not None:
                g_main.replay()
                done += chunk
            if g_tail is not None:
                g_tail.replay()
                done += tail
            if done >= warmup:
                break
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.time()
        e0.record(stream)
        for _ in range(n_full):
            g_main.replay()
        if g_tail is not None:
            g_tail.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        self.windows.append((t0, time.time()))
        barrier()
        return reduce_max(e0.elapsed_time(e1)) / steps  # ms per step

    def release(self):
        self.graphs = []


def auto_steps(est_ms, target_ms=400.0, lo=20, hi=20000):
    return int(min(hi, max(lo, target_ms / max(est_ms, 1e-4))))


def estimate_ms(step):
    import torch
    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(5):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 5


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name):
    """DRAM bytes per launch from a committed ncu summary (a line
    `dram_bytes_per_launch: N` in profiles/<name>.md), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", name + ".md")) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


def roofline(cfg, N, ms, world, kernel, prof):
    peaks = load_peaks()
    _, alg, ops_ = step_units(cfg, N)
    sec = ms / 1e3
    if cfg["metric"] == "TOPS":
        a = ops_ / sec / 1e12
        r = {"bound": "tensor", "achieved": a, "peak": peaks["bf16_tflops"] * world, "unit": "TFLOP/s",
             "peak_note": f"dense bf16 TFLOP/s x {world} GPU(s), {peaks['source']} burst figure (the kernel "
                          f"issues f16 tcgen05 MMAs; f16 dense measured within 3% of bf16 on B200)",
             "frac_of_sustained": a / (peaks["bf16_tflops_sustained"] * world)}
    else:
        a = alg / sec / 1e9
        r = {"bound": "hbm", "achieved": a, "peak": peaks["hbm_gbs"] * world, "unit": "GB/s",
             "peak_note": f"HBM copy bandwidth x {world} GPU(s), {peaks['source']}"}
    r["frac"] = r["achieved"] / r["peak"]
    r["traffic"] = profile_traffic(prof) if world == 1 else None
    r["kernel"] = kernel
    r["algorithmic_bytes_per_step"] = alg
    r["timing"] = "per-step device time over CUDA-graph-replayed steps (all kernels of the step, launch gaps included)"
    return r


# ---------------------------------------------------------------------------
# Single-GPU workloads (kernel-level API on device-resident inputs)
# ---------------------------------------------------------------------------
def mul_mat_case(cfg, N, timer, steps, warmup):
    """Device-timed mul_mat of one config; returns (ms per step, weights, x)."""
    import torch
    from feml_b200 import DType, ops
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    w0 = device_weights(cfg, [0])[0]
    wbytes = w0.numel()
    copies = max(1, math.ceil(2.5 * L2_BYTES / wbytes))
    wts = [w0] + [w0.clone() for _ in range(copies - 1)]
    if dt == DType.F32:
        wts = [w.view(torch.float32).view(M, K) for w in wts]
    x = torch.from_numpy(host_x(cfg, N)).cuda()
    outs = [torch.empty((N, M), dtype=torch.float32, device="cuda") for _ in range(2)]
    wsz = ops.mul_mat_workspace(dt, K, M, N)
    work = torch.empty(max(wsz, 1), dtype=torch.uint8, device="cuda") if wsz else None

    def step(i):
        ops.mul_mat(dt, wts[i % copies], x, K, out=outs[i % 2], workspace=work)

    if steps is None:
        steps = auto_steps(estimate_ms(step))
    ms = timer.run(step, steps, warmup, chunk_hint=copies)
    return ms, steps, copies, wts[0], x


def mul_mat_kernels_per_step(cfg, N):
    from feml_b200 import DType, ops
    return ops.mul_mat_launches(DType[cfg["wtype"]], cfg["K"], cfg["M"], N)


def mul_mat_id_kernels_per_step(cfg, N):
    """Routing, activation quantization and the grouped GEMM, plus the tail
    reduction when the GEMM's largest tile grid (weight-row tiles x the
    column-tile bound) overflows one wave of CTAs (one per SM)."""
    import torch
    bn = 192 if cfg["wtype"] in ("Q8_0", "Q4_0") or (cfg["wtype"] == "Q4_K" and cfg["K"] % 512 == 0) else 128
    max_tiles = -(-N * cfg["n_sel"] // bn) + cfg["E"]
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return 3 + (1 if -(-cfg["M"] // 128) * max_tiles > sms else 0)


def dominant_kernel(cfg, N):
    wt = cfg["wtype"]
    if "E" in cfg:
        return "gemm_tc3_kernel (grouped, tcgen05 split-f16)" if wt in ("Q8_0", "Q4_0") else \
            "gemm_tc_kernel (grouped, tcgen05)"
    if wt == "F32":
        return "gemm_f32_pipe_kernel"
    if N <= 8:
        if wt == "Q4_K" and 12288 <= cfg["K"] <= 16384:
            return "gemv_ks_kernel" if N == 1 else "gemv_ks_cols_kernel"
        return "gemv_kernel"
    split = wt in ("Q8_0", "Q4_0") or (wt == "Q4_K" and cfg["K"] % 512 == 0)
    return "gemm_tc3_kernel (tcgen05 split-f16)" if split else "gemm_tc_kernel (tcgen05)"


def compute_dtype(cfg, N):
    """The arithmetic the dominant kernel computes in."""
    wt = cfg["wtype"]
    if wt == "F32":
        return "f32"
    if N <= 8:
        return "int8 dot / f32 scale"
    if wt in ("Q8_0", "Q4_0") or (wt == "Q4_K" and cfg["K"] % 512 == 0):
        return "f16 hi+lo operands (exact), f32 accumulate"
    return "f16 integer dot / f32 scale"


def mul_mat_id_case(cfg, N, timer, steps, warmup):
    import torch
    from feml_b200 import DType, ops
    dt = DType[cfg["wtype"]]
    K, M, E, n_sel = cfg["K"], cfg["M"], cfg["E"], cfg["n_sel"]
    w0 = device_weights(cfg, list(range(E)))
    copies = max(1, math.ceil(2.5 * L2_BYTES / w0.numel()))
    wts = [w0] + [w0.clone() for _ in range(copies - 1)]
    x = torch.from_numpy(host_x(cfg, N)).cuda()
    ids = torch.from_numpy(host_ids(cfg, N)).cuda()
    outs = [torch.empty((N, n_sel, M), dtype=torch.float32, device="cuda") for _ in range(2)]
    work = torch.empty(ops.mul_mat_id_workspace(dt, K, M, N, n_sel, E), dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def step(i):
        ops.mul_mat_id(dt, wts[i % copies], x, ids, K, out=outs[i % 2], workspace=work, status=status)

    if steps is None:
        steps = auto_steps(estimate_ms(step))
    ms = timer.run(step, steps, warmup, chunk_hint=copies)
    assert int(status.item()) == 0
    return ms, steps, copies, w0


def e2e_c_abi(cfg, N, w_dev, steps, warmup, local):
    """The metric through the reference-facing C ABI with host buffers."""
    import torch
    import feml_b200 as F
    from feml_b200 import DType, GraphBuilder
    K, M = cfg["K"], cfg["M"]
    is_moe = "E" in cfg
    dt = DType[cfg["wtype"]]
    be = F.B200Backend.open(local)
    w_host = w_dev.cpu().numpy()
    g = GraphBuilder()
    if is_moe:
        w = g.weight("w", dt, [K, M, cfg["E"]])
        xi = g.input("x", DType.F32, [K, N])
        ii = g.input("ids", DType.I32, [cfg["n_sel"], N])
        o = g.mul_mat_id(w, xi, ii, cfg["n_sel"])
    else:
        w = g.weight("w", dt, [K, M])
        xi = g.input("x", DType.F32, [K, N])
        ii = None
        o = g.mul_mat(w, xi)
    g.mark_output(o)
    plan = g.compile(be)
    plan.write_tensor(be, w, w_host.reshape(-1).view(np.uint8))
    x_host = torch.from_numpy(host_x(cfg, N)).pin_memory()
    ids_host = torch.from_numpy(host_ids(cfg, N)).pin_memory() if is_moe else None
    y_elems = N * M * (cfg["n_sel"] if is_moe else 1)
    y_host = torch.empty(y_elems, dtype=torch.float32).pin_memory()
    px, po = plan.find(xi), plan.find(o)
    pi = plan.find(ii) if is_moe else None
    x_bytes, y_bytes = N * K * 4, y_elems * 4
    i_bytes = ids_host.numel() * 4 if is_moe else 0

    def one():
        be.write_ptr(plan.buffers[px.buffer].handle, px.offset, x_host.data_ptr(), x_bytes)
        if is_moe:
            be.write_ptr(plan.buffers[pi.buffer].handle, pi.offset, ids_host.data_ptr(), i_bytes)
        be.graph_compute(plan)
        be.read_ptr(plan.buffers[po.buffer].handle, po.offset, y_host.data_ptr(), y_bytes)

    for _ in range(max(3, warmup)):
        one()
    be.synchronize()
    if steps is None:  # about half a second of end-to-end steps
        t0 = time.perf_counter()
        for _ in range(3):
            one()
        steps = int(min(2000, max(10, 0.5 / ((time.perf_counter() - t0) / 3))))
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    be.synchronize()
    dt_s = (time.perf_counter() - t0) / steps
    plan.release(be)
    be.close()
    v, unit = metric_value(cfg, N, dt_s)
    return {"value": v, "unit": unit, "h2d_bytes_per_step": x_bytes + i_bytes, "d2h_bytes_per_step": y_bytes,
            "steps": steps, "ms_per_step": dt_s * 1e3,
            "path": "GraphBuilder->compile->write(pinned x" + (", ids" if is_moe else "") +
                    ")->graph_compute->read(pinned y), libfeml_b200 C ABI"}


def extra_line(name, cfg, N, ms, steps, copies, world=1, e2e=None):
    v, unit = metric_value(cfg, N, ms / 1e3)
    r = roofline(cfg, N, ms, world, dominant_kernel(cfg, N), f"{name}_{cfg['wtype'].lower()}_n{N}")
    d = {"metric": metric_name(name, cfg), "value": v, "unit": unit, "ms_per_step": ms, "steps": steps,
         "N": N, "roofline_frac": r["frac"], "roofline": r,
         "l2": f"{copies} rotating weight copies" if copies > 1 else "weights larger than 2x L2"}
    if e2e is not None:
        d["e2e"] = e2e
    return d


def run_extras_single(args, timer):
    """The other workloads of the path on this GPU (N=1 only)."""
    import torch
    out, launches = {}, 0
    todo = [("c2", 1), ("c3", 512), ("c4", 1), ("c4", 8), ("c4", 64), ("c1", 32)]
    for name, N in todo:
        cfg = CONFIGS[name]
        ms, steps, copies, w0, _ = mul_mat_case(cfg, N, timer, None, args.warmup)
        e2e = None
        if name == "c2":
            e2e = e2e_c_abi(cfg, N, w0, None, args.warmup, torch.cuda.current_device())
        key = f"{name}_n{N}" if name == "c4" else name
        out[key] = extra_line(name, cfg, N, ms, steps, copies, e2e=e2e)
        out[key]["gpu_launches"] = steps * mul_mat_kernels_per_step(cfg, N)
        launches += out[key]["gpu_launches"]
        del w0
        torch.cuda.empty_cache()
    return out, launches


# ---------------------------------------------------------------------------
# Multi-GPU workloads
# ---------------------------------------------------------------------------
def experts_sharded_case(cfg, N, timer, steps, warmup, combine, e2e_steps):
    """C5 expert-sharded across the ranks with the given combine."""
    import torch
    from feml_b200 import DType
    from feml_b200.shard import ExpertShardedMulMatId
    import torch.distributed as dist
    rank, ws = dist.get_rank(), dist.get_world_size()
    dt = DType[cfg["wtype"]]
    K, E, n_sel = cfg["K"], cfg["E"], cfg["n_sel"]
    mine = [e for e in range(E) if e % ws == rank]
    w_local = device_weights(cfg, mine)
    copies = max(1, math.ceil(2.5 * L2_BYTES / max(w_local.numel(), 1)))
    wts = [w_local] + [w_local.clone() for _ in range(copies - 1)]
    x = torch.from_numpy(host_x(cfg, N)).cuda()
    ids = torch.from_numpy(host_ids(cfg, N)).cuda()
    fused = combine in ("owner", "replicate")
    mod = ExpertShardedMulMatId(dt, wts[0], K, E, local=True, fused=fused, max_tokens=N, max_selected=n_sel,
                                combine="owner" if combine == "owner" else "replicate")

    def step(i):
        mod.w_local = wts[i % copies]
        return mod(x, ids)

    if steps is None:
        steps = auto_steps(reduce_max(estimate_ms(step)))
    ms = timer.run(step, steps, warmup, chunk_hint=copies)
    e2e = None
    if e2e_steps:
        lo, hi = mod.token_range(N) if combine == "owner" else (0, N)
        x_host = torch.from_numpy(host_x(cfg, N)).pin_memory()
        ids_host = torch.from_numpy(host_ids(cfg, N)).pin_memory()
        y_host = torch.empty((hi - lo) * n_sel * cfg["M"], dtype=torch.float32).pin_memory()

        def one(i):
            x.copy_(x_host, non_blocking=True)
            ids.copy_(ids_host, non_blocking=True)
            y_host.copy_(step(i).reshape(-1), non_blocking=True)

        for i in range(max(3, warmup)):
            one(i)
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            one(i)
        torch.cuda.synchronize()
        e2e_s = reduce_max(time.perf_counter() - t0) / e2e_steps
        v, unit = metric_value(cfg, N, e2e_s)
        e2e = {"value": v, "unit": unit, "h2d_bytes_per_step": x_host.numel() * 4 + ids_host.numel() * 4,
               "d2h_bytes_per_step": y_host.numel() * 4, "steps": e2e_steps, "ms_per_step": e2e_s * 1e3,
               "path": "feml_b200.shard.ExpertShardedMulMatId: pinned host x, ids -> device -> "
                       + ("this rank's tokens' slots" if combine == "owner" else "all slots") + " -> pinned host"}
    torch.cuda.synchronize()
    barrier()
    mod.close()
    # route + quantize + grouped GEMM, then the flag wait (peer-store
    # combines) or the tail reduction when the tile grid overflows a wave
    kernels = 3 + (1 if fused else mul_mat_id_kernels_per_step(dict(cfg, E=len(mine)), N) - 3)
    return ms, steps, copies, e2e, kernels


def rows_sharded_case(cfg, N, timer, warmup, fused):
    """C4 row-sharded decode step (GEMV on this rank's rows + the combine)."""
    import torch
    from feml_b200 import DType
    from feml_b200.shard import RowShardedMulMat, row_range
    import torch.distributed as dist
    rank, ws = dist.get_rank(), dist.get_world_size()
    dt = DType[cfg["wtype"]]
    K, M = cfg["K"], cfg["M"]
    lo, hi, _ = row_range(M, rank, ws)
    w_local = device_weights(cfg, [0], rows=(lo, hi))[0]
    copies = max(1, math.ceil(2.5 * L2_BYTES / max(w_local.numel(), 1)))
    wts = [w_local] + [w_local.clone() for _ in range(copies - 1)]
    x = torch.from_numpy(host_x(cfg, N)).cuda()
    mod = RowShardedMulMat(dt, wts[0], K, M, local=True, fused=fused)

    def step(i):
        mod.w_local = wts[i % copies]
        return mod(x)

    steps = auto_steps(reduce_max(estimate_ms(step)))
    ms = timer.run(step, steps, warmup, chunk_hint=copies)
    torch.cuda.synchronize()
    barrier()
    mod.close()
    return ms, steps, copies


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm
# ---------------------------------------------------------------------------
def cpu_sample(cfg, N, rows, threads, seconds_budget, max_iters=1000):
    """The reference's CPU mul_mat (oracle/: feml-cpu/src/ops/mul_mat.rs:36-57
    restated in C) on the first `rows` weight rows of every expert and every
    output column. The reference has no quantized kernel: its path is the F32
    mul_mat on the dequantized weights and, as on the device, Q8_0-rounded
    activations. Returns seconds per full step (scaled by M / rows)."""
    once = reference_sampler(cfg, N, rows, threads)
    once()
    t_end = time.perf_counter() + seconds_budget
    n, tx, tm = 0, 0.0, 0.0
    while True:
        a, b = once()
        tx, tm = tx + a, tm + b
        n += 1
        if time.perf_counter() > t_end or n >= max_iters:
            break
    return (tx + tm * (cfg["M"] / rows)) / n, n, tx + tm


def sample_rows(cfg, N, macs):
    n_cols = N * cfg.get("n_sel", 1)
    return int(min(cfg["M"], max(8, macs // (cfg["K"] * n_cols))))


def cpu_baseline(cfg, N, budget_s):
    rows = sample_rows(cfg, N, 1.5e8)
    n_cols = N * cfg.get("n_sel", 1)
    sec1, n1, t1 = cpu_sample(cfg, N, rows, 1, budget_s)
    threads = os.cpu_count() or 1
    secm, nm, tm = cpu_sample(cfg, N, rows, threads, budget_s / 2)
    v1, unit = metric_value(cfg, N, sec1)
    vm, _ = metric_value(cfg, N, secm)
    return {"value": v1, "unit": unit, "cores": 1, "kind": "port",
            "sample": f"{rows}/{cfg['M']} weight rows of every expert x {n_cols} output columns per iteration, "
                      f"{n1} iterations ({t1:.1f} s) on 1 core (the reference executes plans single-threaded, "
                      f"docs/api-guide.md:147); value scaled to the full step",
            "sec_per_full_step": sec1,
            "multi_thread": {"value": vm, "unit": unit, "cores": threads, "iterations": nm,
                             "sec_per_full_step": secm}}


def reference_sampler(cfg, N, rows, threads):
    """A step of the reference's CPU path on the first `rows` weight rows of
    every expert and every output column; returns the callable."""
    from oracle import oracle as O
    K = cfg["K"]
    code = DT_CODE[cfg["wtype"]]
    experts = list(range(cfg.get("E", 1)))
    wdeq = []
    for e in experts:
        wf = host_weight_rows(cfg, e, 0, rows)
        wdeq.append(wf if cfg["wtype"] == "F32" else O.dequantize(code, O.quantize(code, wf), K))
    x = host_x(cfg, N)
    if "E" in cfg:
        ids = host_ids(cfg, N)
        groups = [(e, np.nonzero((ids == e).any(axis=1))[0]) for e in experts]
    else:
        groups = [(0, np.arange(N))]

    def sample():
        """(seconds rounding the activations -- once per full step, not scaled
        by the row sample -- and seconds of the sampled mul_mat rows)."""
        t0 = time.perf_counter()
        xf = x if cfg["wtype"] == "F32" else O.dequantize(O.DT_Q8_0, O.quantize(O.DT_Q8_0, x), K)
        t1 = time.perf_counter()
        for e, toks in groups:
            if len(toks):
                O.mul_mat_f32(wdeq[e], xf[toks], nthreads=threads)
        return t1 - t0, time.perf_counter() - t1

    return sample


def run_reference(args, cfg_name, cfg, N):
    """The reference's CPU mul_mat on all host threads (the oracle port; the
    Rust reference cannot be built here). Each step is a bounded sample of
    the workload (the first weight rows of every expert, all output
    columns), sized from a calibration run so the whole run takes about a
    minute and a half; the value is scaled to the full step. Imports nothing
    from feml_b200."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    M = cfg["M"]
    threads = os.cpu_count() or 1
    total_steps = args.steps + args.warmup
    probe_rows = min(M, 16)
    probe = reference_sampler(cfg, N, probe_rows, threads)
    probe()
    t_x, t_mm = probe()
    per_row = t_mm / probe_rows
    target = min(2.0, max(0.05, 90.0 / total_steps))  # seconds per sample step
    rows = int(min(M, max(probe_rows, (target - t_x) / max(per_row, 1e-9))))
    sample = reference_sampler(cfg, N, rows, threads)
    for _ in range(args.warmup):
        sample()
    tx = tm = 0.0
    for _ in range(args.steps):
        a, b = sample()
        tx, tm = tx + a, tm + b
    sec_full = (tx + tm * (M / rows)) / args.steps
    v, unit = metric_value(cfg, N, sec_full)
    n_cols = N * cfg.get("n_sel", 1)
    print(json.dumps({
        "impl": "reference", "metric": metric_name(cfg_name, cfg), "value": v, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec_full * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy draws shared with the GPU arm)",
        "config": config_dict(cfg_name, cfg, N, world),
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"{rows}/{M} weight rows of every expert x {n_cols} output columns per step, "
                                   f"scaled to the full step; F32 mul_mat (feml-cpu/src/ops/mul_mat.rs:36-57 "
                                   f"restated in C) on dequantized weights and Q8_0-rounded activations"},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
def run_b200(args, cfg_name, cfg, N):
    import torch
    ws, rank, local = dist_setup()
    windows = []
    timer = Timer(windows)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    is_moe = "E" in cfg
    extras = {}
    if ws == 1:
        if is_moe:
            ms, steps, copies, w0 = mul_mat_id_case(cfg, N, timer, args.steps, args.warmup)
            launches = steps * mul_mat_id_kernels_per_step(cfg, N)
        else:
            ms, steps, copies, w0, _ = mul_mat_case(cfg, N, timer, args.steps, args.warmup)
            launches = steps * mul_mat_kernels_per_step(cfg, N)
        e2e = e2e_c_abi(cfg, N, w0, args.e2e_steps, args.warmup, local)
        del w0
        torch.cuda.empty_cache()
        if not args.no_extras:
            extras, _ = run_extras_single(args, timer)  # each extra line carries its own count
        scaling = "strong"
    else:
        if not is_moe:
            raise SystemExit("the multi-GPU headline is the expert-sharded C5 (--config c5)")
        ms, steps, copies, e2e, k = experts_sharded_case(cfg, N, timer, args.steps, args.warmup, args.combine,
                                                         args.e2e_steps or 50)
        launches = steps * k
        if not args.no_extras:
            for comb in [c for c in ("owner", "replicate", "nccl") if c != args.combine]:
                ms_c, st_c, cp_c, _, k_c = experts_sharded_case(cfg, N, timer, None, args.warmup, comb, 0)
                extras[f"c5_{comb}"] = extra_line("c5", cfg, N, ms_c, st_c, cp_c, world=ws)
                extras[f"c5_{comb}"]["combine"] = comb
                extras[f"c5_{comb}"]["gpu_launches"] = st_c * k_c
            c4 = CONFIGS["c4"]
            ms_r, st_r, cp_r = rows_sharded_case(c4, 1, timer, args.warmup, fused=True)
            extras["c4_rows_fused_n1"] = extra_line("c4", c4, 1, ms_r, st_r, cp_r, world=ws)
            extras["c4_rows_fused_n1"]["gpu_launches"] = st_r * 2
        scaling = "strong"
    time.sleep(0.25)
    sampler.stop()
    clocks = sampler.summary(windows)
    value, unit = metric_value(cfg, N, ms / 1e3)
    result = {
        "metric": metric_name(cfg_name, cfg), "value": value, "unit": unit, "n_gpus": ws, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": compute_dtype(cfg, N),
        "data": "synthetic (seeded numpy draws, quantized on device by the library's quantizer)",
        "config": config_dict(cfg_name, cfg, N, ws),
        "l2": f"{copies} rotating weight copies per rank" if copies > 1 else "weights larger than 2x L2 per rank",
        "combine": None if ws == 1 else args.combine,
        "roofline": roofline(cfg, N, ms, ws, dominant_kernel(cfg, N), f"{cfg_name}_{cfg['wtype'].lower()}_n{N}"),
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks,
        "extras": extras,
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg, N, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)
    timer.release()  # graphs go before the process group
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: about half a second of work)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    ap.add_argument("--tokens", type=int, default=None, help="activation columns N (c4: 1, 8 or 64)")
    ap.add_argument("--combine", default="owner", choices=["owner", "replicate", "nccl"],
                    help="C5 on N>1 GPUs: slots to their token's owner rank (peer stores), to every rank (peer "
                         "stores), or an NCCL all-reduce")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = dict(CONFIGS[args.config])
    N = args.tokens if args.tokens is not None else cfg["N"]
    if args.impl == "reference":
        if args.steps is None:
            args.steps = 20
        run_reference(args, args.config, cfg, N)
        return
    run_b200(args, args.config, cfg, N)


if __name__ == "__main__":
    main()
