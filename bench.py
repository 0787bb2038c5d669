"""Benchmark of the acediaR tensor hot path on B200.

Default workload (the configuration quoted at 1/2/4/8 GPUs): a float32
256 x 512 x 32768 tensor (2^32 elements, 16 GiB, N(0,1)), sharded along its
outermost axis, one step =
    y <- contiguous(permute_view(x, c(3,1,2)))      # one kernel (acd_permute_fused_stats_keys):
    z <- y*0.5 + exp(-y^2)                          #   x read once, y and z written once,
    sum(z), var(z)                                  #   with the shard's statistics row
    argmax(z, axis = 1)                             #   and argmax keys
then one int64 MAX all-reduce of keys and rows (N > 1) and the finish kernel
(rows merged in rank order, keys decoded).  The metric is Gelem/s of the
whole job (2^32 / step time, max over ranks).  The one-GPU line also carries
the per-op reports of the other four configurations (per_config).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Under torchrun each rank drives one GPU (NCCL).  --impl reference times the
CPU restatement of the same step (all host threads) on a bounded sample.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "acedia-r_b200"))

N0, N1, N2 = 256, 512, 32768
CHUNK = 128  # shards hold whole multiples of 128 slices along axis 3
SEED = 42
CPU_SAMPLE_N2 = 2048  # CPU baseline sample: 256 x 512 x 2048 (2^28 elements)
# algorithmic bytes per element of the step kernel: x read, y and z written (4 B each)
BYTES_PER_ELEM = {"permute_chain_stats_keys": 12}
# DRAM bytes per element that ncu measured (dram__bytes_read.sum + dram__bytes_write.sum, mean of 10
# launches) on the 256x512x1024 case of the same step, scaled by elements to a full launch.  Reads are
# exactly 4 B/elem; the write side reads low by the ~58 MB of dirty lines still in L2 when a launch ends.
TRAFFIC_BYTES_PER_ELEM = {"permute_chain_stats_keys": 11.568}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="acediar", choices=["acediar", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--n2", type=int, default=N2, help="extent of the sharded axis (default 32768)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per-op reports of the other configurations on the default one-GPU run")
    ap.add_argument("--workload", default="views", choices=["views", "c1", "c2", "c3", "c4"],
                    help="views (default, the sharded strided-views step) or a per-op report of one of the "
                         "other configurations on one GPU")
    ap.add_argument("--only", default=None,
                    help="per-op reports: time only the ops whose name contains this text (e.g. 'var(T, axis=2)')")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """Samples SM clocks and throttle reasons during the timed region."""

    def __init__(self, devices):
        self.devices = set(devices)
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()  # wait for the sampler's first line before timing
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                if int(f[0]) not in self.devices:
                    continue
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
def reference_arm(a):
    """CPU restatement of the step on all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = os.cpu_count() or 1
    n2 = CPU_SAMPLE_N2
    rng = np.random.default_rng(SEED)
    x = rng.standard_normal(N0 * N1 * n2, dtype=np.float32)
    y = np.empty_like(x)
    z = np.empty_like(x)
    idx = np.empty(N0 * N1, dtype=np.int32)
    for _ in range(a.warmup):
        oracle.pipeline_views_raw(x, N0, N1, n2, y, z, idx, threads)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        oracle.pipeline_views_raw(x, N0, N1, n2, y, z, idx, threads)
    dt = (time.perf_counter() - t0) / a.steps
    n = N0 * N1 * n2
    v = n / dt / 1e9
    line = {
        "metric": "Gelem/s, strided-views step (permute->contiguous, x*0.5+exp(-x^2), sum/var, argmax axis 1)",
        "value": round(v, 4), "unit": "Gelem/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic N(0,1), numpy PCG64 seed 42 (the CPU sample; the GPU arm uses acd_rand)",
        "config": {"workload": "strided views 256x512x32768 f32 (CPU sample 256x512x%d)" % n2,
                   "l2": "inputs larger than L2"},
        "impl": "reference",
        "cpu_baseline": {"value": round(v, 4), "unit": "Gelem/s", "cores": threads, "kind": "port",
                         "sample": "256x512x%d f32 (2^28 elements), same step, base-R-equivalent double math" % n2},
        "e2e": {"value": round(v, 4), "unit": "Gelem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_single(sample_n2=256):
    """Single-thread oracle timing on a bounded sample (Gelem/s)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    rng = np.random.default_rng(SEED)
    n = N0 * N1 * sample_n2
    x = rng.standard_normal(n, dtype=np.float32)
    y, z = np.empty_like(x), np.empty_like(x)
    idx = np.empty(N0 * N1, dtype=np.int32)
    oracle.pipeline_views_raw(x, N0, N1, sample_n2, y, z, idx, 1)
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.pipeline_views_raw(x, N0, N1, sample_n2, y, z, idx, 1)
        reps += 1
        if time.perf_counter() - t0 > 8.0:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(n / dt / 1e9, 4), "unit": "Gelem/s", "cores": 1, "kind": "port",
            "sample": "256x512x%d f32 (%d elements), single thread, %d reps" % (sample_n2, n, reps)}


# ---------------------------------------------------------------------------
# per-op reports of the other configurations (one GPU)
# ---------------------------------------------------------------------------
def _time(fn, reps=10, warm=3):
    import torch
    for _ in range(warm):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _time_graph(fn, reps=10, replays=5):
    """Device time of one call: `reps` calls captured once in a CUDA graph and
    replayed, so per-call host overhead (the Python wrapper) is not counted.
    Only for calls that never synchronise with the host."""
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                fn()
    torch.cuda.synchronize()
    graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(replays):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / (replays * reps)


_ONLY = None  # --only: time just the ops whose name contains this text


def _op(name, fn, nbytes, peak, reps=10, note=None, graph=False):
    """Times `fn`.  graph=True (calls that return device tensors) reports the
    device time from CUDA-graph replay as `ms` and the eager per-call time,
    host wrapper included, as `eager_ms`.  Returns None for an op that --only
    leaves out."""
    if _ONLY is not None and _ONLY not in name:
        return None
    eager = _time(fn, reps)
    ms = _time_graph(fn, reps) if graph else eager
    gbs = nbytes / (ms * 1e-3) / 1e9
    d = {"op": name, "ms": round(ms, 4), "bytes": int(nbytes), "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4)}
    if graph:
        d["eager_ms"] = round(eager, 4)
    if note:
        d["note"] = note
    return d


def config_ops(workload, peak):
    """(workload description, op records) of one configuration's per-op report
    on the current GPU (c1, c2, c3 or c4)."""
    import numpy as np
    import torch

    import acediar as acd
    import acediar._lib as L
    import acediar.tensor as Tm

    g = torch.Generator(device="cuda")
    g.manual_seed(SEED)
    ops = []
    if workload == "c1":
        n = 1 << 20
        ta = acd.from_torch(torch.rand(n, generator=g, device="cuda", dtype=torch.float64), (n,), "double")
        tb = acd.from_torch(torch.randn(n, generator=g, device="cuda", dtype=torch.float64), (n,), "double")
        B = 8 * n
        ops.append(_op("a+b", lambda: ta + tb, 3 * B, peak, graph=True))
        ops.append(_op("a*b", lambda: ta * tb, 3 * B, peak, graph=True))
        ops.append(_op("exp(a)", lambda: acd.exp(ta), 2 * B, peak, graph=True))
        ops.append(_op("sigmoid(b)", lambda: acd.sigmoid(tb), 2 * B, peak, graph=True))
        ops.append(_op("sqrt(a)", lambda: acd.sqrt(ta), 2 * B, peak, graph=True))
        c = ta + tb
        ops.append(_op("sum(c)", lambda: acd.tensor_sum(c), B, peak, graph=True))
        ops.append(_op("var(c)", lambda: acd.tensor_var(c), B, peak, graph=True))
        ops.append(_op("which.max(c)", lambda: Tm._arg("argmax", c), B, peak, graph=True))

        def config():
            c_ = ta + tb
            d_ = ta * tb
            e_ = acd.exp(ta)
            f_ = acd.sigmoid(tb)
            g_ = acd.sqrt(ta)
            outs = []
            for t in (c_, d_, e_, f_, g_):
                outs += [acd.tensor_sum(t), acd.tensor_mean(t), acd.tensor_var(t)]
            return outs
        total_bytes = 3 * B * 2 + 2 * B * 3 + 15 * B + B
        ops.append(_op("whole config (eager)", config, total_bytes, peak, note="20 launches, L2-resident 8 MiB arrays"))
        # the same 20 launches captured once in a CUDA graph and replayed
        for _ in range(3):
            config()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                config()
        torch.cuda.synchronize()
        ops.append(_op("whole config (CUDA graph)", graph.replay, total_bytes, peak, reps=50,
                       note="launch overhead removed; arrays stay in L2"))
        # one kernel: a and b read once, c..g written once, 15 statistics and
        # which.max from the same registers (56 MiB moved)
        ops.append(_op("whole config (one kernel, acd_chain5_stats)", lambda: Tm.chain5_stats(ta, tb), 7 * B, peak,
                       graph=True, reps=20, note="algorithmic bytes: a, b read + c..g written"))
        workload = "elementwise chain + reductions, float64 n=2^20"
        unit_elems = n
    elif workload == "c2":
        R = C = 8192
        X = acd.from_torch(torch.randn(R * C, generator=g, device="cuda"), (R, C), "float")
        r = acd.from_torch(torch.rand(C, generator=g, device="cuda") * 2 - 1, (1, C), "float")
        B = 4 * R * C
        Y = acd.fused("add_relu", X, r)
        M = X > r
        ops.append(_op("relu(X+r) fused", lambda: acd.fused("add_relu", X, r), 2 * B, peak, graph=True))
        ops.append(_op("X+r", lambda: X + r, 2 * B, peak, graph=True))
        ops.append(_op("X>r -> bool", lambda: X > r, B + R * C, peak, graph=True))
        ops.append(_op("pmax(X,r)", lambda: acd.pmax(X, r), 2 * B, peak, graph=True))
        ops.append(_op("tanh(X)*2 fused", lambda: acd.fused("tanh_scale", X, p0=2.0), 2 * B, peak, graph=True))
        ops.append(_op("colSums(Y)", lambda: acd.tensor_sum(Y, axis=[1]), B, peak, graph=True))
        ops.append(_op("count(M) per column", lambda: acd.tensor_count(M, axis=[1]), R * C, peak, graph=True))
        workload = "broadcast + compare, float32 8192x8192 + 1x8192"
        unit_elems = R * C
    elif workload == "c3":
        shp = (4096, 4096, 16)
        n = 4096 * 4096 * 16
        T = acd.from_torch(torch.randn(n, generator=g, device="cuda"), shp, "float")
        I = acd.from_torch(torch.randint(-1000, 1001, (n,), generator=g, device="cuda", dtype=torch.int32), shp, "int32")
        B = 4 * n
        for op in ("sum", "mean", "var", "max"):
            ops.append(_op("%s(T)" % op, (lambda op=op: getattr(acd, "tensor_" + op)(T)), B, peak))
        sv_s, sv_v = Tm._alloc((1,), "double"), Tm._alloc((1,), "double")
        sv_d = (sv_s.desc(), sv_v.desc(), T.desc())

        def sum_var_device():
            L.check(L.lib().acd_sum_var(Tm.context(), ctypes.byref(sv_d[0]), ctypes.byref(sv_d[1]),
                                        ctypes.byref(sv_d[2]), Tm._stream()), "sum_var")
        ops.append(_op("sum+var fused", sum_var_device, B, peak, graph=True,
                       note="device outputs; acd.sum_var() adds two 8-byte host reads"))
        ops.append(_op("sum+var fused, host result", lambda: acd.sum_var(T), B, peak,
                       note="includes two synchronising 8-byte D2H reads"))
        ops.append(_op("which.max(T)", lambda: Tm._arg("argmax", T), B, peak))
        ops.append(_op("as.double(T)", lambda: acd.to_dtype(T, "double"), B + 2 * B, peak, graph=True))
        ops.append(_op("rnorm_tensor(4096x4096x16)", lambda: acd.rnorm_tensor(shp), B, peak, graph=True,
                       note="Philox4x32-10 + Box-Muller, write-only"))
        ops.append(_op("rand_tensor(4096x4096x16)", lambda: acd.rand_tensor(shp), B, peak, graph=True))
        ops.append(_op("as.integer(T)", lambda: acd.to_dtype(T, "int32"), 2 * B, peak, graph=True))
        for ax in (1, 2, 3):
            kept = n // shp[ax - 1]
            for op in ("sum", "mean", "var", "max"):
                ops.append(_op("%s(T, axis=%d)" % (op, ax), (lambda op=op, ax=ax: getattr(acd, "tensor_" + op)(T, axis=[ax])),
                               B + 4 * kept, peak))
            ops.append(_op("argmax(T, axis=%d)" % ax, (lambda ax=ax: acd.argmax(T, axis=ax)), B + 8 * kept, peak))
        ops.append(_op("sum(int32 T)", lambda: acd.tensor_sum(I), B, peak))
        U = acd.from_torch(torch.rand(64 * 1048576, generator=g, device="cuda"), (64, 1048576), "float")
        ops.append(_op("cumsum(U, axis=2)", lambda: acd.cumsum(U, axis=2), 2 * 4 * 64 * 1048576, peak))
        workload = "axis reductions float32 4096x4096x16, int32 sum, cumsum 64x1048576"
        unit_elems = n
    else:
        R, C = 65536, 4096
        Xf = acd.from_torch(torch.randn(R * C, generator=g, device="cuda") * 2.0, (R, C), "float")
        off = acd.from_torch(torch.rand(R, generator=g, device="cuda") * 100 - 50, (R, 1), "float")
        Xf = Xf + off
        ops.append(_op("softmax f32 65536x4096 axis=2", lambda: acd.softmax(Xf, axis=2), 2 * 4 * R * C, peak))
        R2, C2 = 1024, 32768
        Xd = acd.from_torch(torch.randn(R2 * C2, generator=g, device="cuda", dtype=torch.float64), (R2, C2), "double")
        ops.append(_op("softmax f64 1024x32768 axis=2", lambda: acd.softmax(Xd, axis=2), 2 * 8 * R2 * C2, peak))
        ops.append(_op("softmax f32 whole tensor", lambda: acd.softmax(Xf), 3 * 4 * R * C, peak))
        if _ONLY is None or _ONLY in "row sums of f32 softmax":
            sm = acd.softmax(Xf, axis=2)
            rows = acd.tensor_sum(sm, axis=[2]).as_array()
            ops.append({"op": "row sums of f32 softmax", "max_abs_dev_from_1": float(np.abs(rows - 1).max())})
        workload = "row softmax float32 65536x4096 (N(0,4) + row offset U(-50,50)), float64 1024x32768"
        unit_elems = R * C
    del unit_elems
    return workload, [o for o in ops if o is not None]


def run_config_report(a):
    import torch

    global _ONLY
    _ONLY = a.only
    torch.cuda.set_device(0)
    peak, peak_kind = peaks()
    workload, ops = config_ops(a.workload, peak)
    line = {"metric": "HBM GB/s per op (algorithmic bytes / CUDA-event time)", "workload": workload,
            "peak_GB/s": peak, "peak_source": peak_kind, "ops": ops, "n_gpus": 1}
    print(json.dumps(line), flush=True)


def per_config_block(peak):
    """The per-op reports of the four other configurations, compact, for the
    default one-GPU line: op -> [device ms, fraction of the HBM peak]."""
    import torch
    out = {}
    for w in ("c1", "c2", "c3", "c4"):
        workload, ops = config_ops(w, peak)
        out[w] = {"workload": workload,
                  "ops": {o["op"]: ([o["ms"], o["frac"]] if "ms" in o else {k: v for k, v in o.items() if k != "op"})
                          for o in ops}}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
def main():
    a = parse()
    if a.impl == "reference":
        return reference_arm(a)
    if a.workload != "views":
        return run_config_report(a)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    import acediar
    import acediar._lib as L
    from acediar import sharded as SH
    from acediar.tensor import _alloc, context, gpuTensor

    lib = L.lib()
    ctx = context(local)
    n2 = a.n2
    lo, hi = SH.shard_bounds(n2 // CHUNK, rank, world)
    lo, hi = lo * CHUNK, hi * CHUNK
    n2l = hi - lo
    nloc = N0 * N1 * n2l
    ntot = N0 * N1 * n2

    # ---- input: x[:, :, lo:hi] from this library's counter-based generator:
    # element (a, b, c) is counter position a + 256 (b + 512 c) of seed 42, so
    # every GPU count holds exactly the same tensor
    x = _alloc((N0, N1, n2l), "float", dev)
    L.check(lib.acd_rand(ctx, ctypes.byref(x.desc()), 1, ctypes.c_double(0.0), ctypes.c_double(1.0),
                         ctypes.c_uint64(SEED), ctypes.c_uint64(lo * N0 * N1),
                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "rand")

    # ---- preallocated outputs
    xp_view = acediar.permute_view(x, [3, 1, 2])
    y = _alloc((n2l, N0, N1), "float", dev)
    z = _alloc((n2l, N0, N1), "float", dev)
    # two int64 exchange buffers (steps alternate): the argmax keys, then one
    # statistics row per rank; a single MAX all-reduce carries both
    # (acediar.sharded).  Step k's exchange and finish run on a side stream
    # under step k+1's kernel; step k+2 reuses the buffer once step k's
    # finish has read it.
    nkeys = N0 * N1
    xbufs = [SH.exchange_buffer(nkeys, world, dev) for _ in range(2)]
    row_ptrs = [SH.row_slot(b, nkeys, rank) for b in xbufs]
    keys_ptrs = [ctypes.c_void_p(b.data_ptr()) for b in xbufs]
    side = torch.cuda.Stream(device=dev)
    finished = [None, None]  # events: step's finish has read the buffer
    sum_var = torch.empty(2, dtype=torch.float64, device=dev)
    sv_ptr = ctypes.c_void_p(sum_var.data_ptr())
    idx = _alloc((N0, N1), "int32", dev)
    d_xp, d_y, d_z, d_idx = xp_view.desc(), y.desc(), z.desc(), idx.desc()
    pref = ctypes.byref

    def stream():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def k_step(s, b=0, dx=None):
        # y = contiguous(permute(x)), z = y*0.5 + exp(-y^2), this shard's
        # statistics row of z and the argmax keys of z along axis 1, in one
        # kernel that reads x once; the row and keys go straight into
        # exchange buffer b
        L.check(lib.acd_permute_fused_stats_keys(ctx, pref(d_y), pref(d_z), pref(dx if dx is not None else d_xp),
                                                 ctypes.c_double(0.5), row_ptrs[b], keys_ptrs[b], lo, s),
                "permute_fused_stats_keys")

    def exchange(b=0, async_op=False):
        if world > 1:
            return dist.all_reduce(xbufs[b], op=dist.ReduceOp.MAX, async_op=async_op)
        return None

    def k_finish(s, b=0):
        # argmax indices, and the rows merged in rank order into (sum, var)
        L.check(lib.acd_shard_finish(ctx, keys_ptrs[b], nkeys, world, pref(d_idx), sv_ptr, 1, s), "shard_finish")

    def step(k, dx=None, input_read=None):
        s = stream()
        b = k % 2
        if finished[b] is not None:
            torch.cuda.current_stream().wait_event(finished[b])  # step k-2's finish has read buffer b
        k_step(s, b, dx)
        if input_read is not None:
            input_read.record()  # the step kernel is the only reader of the input
        work = exchange(b, async_op=True)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            if work is not None:
                work.wait()  # the side stream waits for the collective
            k_finish(ctypes.c_void_p(side.cuda_stream), b)
            ev = torch.cuda.Event()
            ev.record(side)
            finished[b] = ev

    def join():
        torch.cuda.current_stream().wait_stream(side)

    LAUNCHES_PER_STEP = 2  # the step kernel, the exchange finish

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for k in range(max(3, a.warmup)):
        step(k)
    join()
    barrier()
    clocks = Clocks([local]) if rank == 0 else None
    if clocks:
        clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for k in range(a.steps):
        step(k)
    join()  # the last step's exchange and finish are inside the timed region
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1) / a.steps
    clk = clocks.stop() if clocks else None
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    result_sum, result_var = (float(v) for v in sum_var.cpu().tolist())
    idx_host = idx.storage[:N0 * N1].cpu()

    # ---- phase split of the step (CUDA events on the launching stream; the
    # synchronous all-reduce makes that stream wait for NCCL's), max over ranks
    PH = 5
    pev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(PH)]
    barrier()
    for k in range(PH):
        pev[k][0].record()
        k_step(stream())
        pev[k][1].record()
        exchange()
        pev[k][2].record()
        k_finish(stream())
        pev[k][3].record()
    barrier()
    names = ["permute_chain_stats_keys", "exchange", "finish"]
    ph = torch.tensor([sum(pev[k][j].elapsed_time(pev[k][j + 1]) for k in range(PH)) / PH for j in range(3)],
                      dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
    phases = {n: round(float(v), 4) for n, v in zip(names, ph.tolist())}
    result_idx = {"checksum": int(idx_host.to(torch.int64).sum().item()), "first": int(idx_host[0].item()),
                  "last": int(idx_host[-1].item())}

    # ---- per-kernel durations (CUDA events on the launching stream)
    kern = {}
    for name, fn in [("permute_chain_stats_keys", k_step)]:
        for _ in range(2):
            fn(stream())
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        reps = 5
        ev[0].record()
        for _ in range(reps):
            fn(stream())
        ev[1].record()
        torch.cuda.synchronize()
        kern[name] = ev[0].elapsed_time(ev[1]) / reps
    # ---- the ceiling of the step's traffic mix: x read once, written to y and
    # to z, as plain contiguous streaming (no transpose, no arithmetic)
    def k_fanout(s):
        L.check(lib.acd_copy_fanout(ctx, ctypes.c_void_p(y.storage.data_ptr()), ctypes.c_void_p(z.storage.data_ptr()),
                                    ctypes.c_void_p(x.storage.data_ptr()), nloc * 4, s), "copy_fanout")

    for _ in range(2):
        k_fanout(stream())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(5):
        k_fanout(stream())
    ev[1].record()
    torch.cuda.synchronize()
    fan_gbs = 12 * nloc / (ev[0].elapsed_time(ev[1]) / 5 * 1e-3) / 1e9
    peak, peak_kind = peaks()
    ops = []
    for name, kms in kern.items():
        byts = BYTES_PER_ELEM[name] * nloc
        gbs = byts / (kms * 1e-3) / 1e9
        tr = TRAFFIC_BYTES_PER_ELEM[name]
        ops.append({"kernel": name, "ms": round(kms, 4), "bytes": byts, "GB/s": round(gbs, 1),
                    "frac": round(gbs / peak, 4), "traffic": int(tr * nloc) if tr else None})
    top = max(ops, key=lambda o: o["ms"])

    # ---- end to end: host buffers in, results out, through the same C ABI.
    # Every step copies its input from pinned host memory and reads its results
    # back.  Two device input buffers let the copy of step k+1 (on a copy
    # stream) run under the kernels of step k: the copy into a buffer waits
    # for the step kernel that last read it, the step waits for its copy.
    e2e = None
    if a.e2e_steps > 0:
        xh = torch.empty(nloc, dtype=torch.float32, pin_memory=True)
        xh.copy_(x.storage[:nloc])
        x2 = _alloc((N0, N1, n2l), "float", dev)
        d_xp2 = acediar.permute_view(x2, [3, 1, 2]).desc()
        bufs = [(x.storage, d_xp), (x2.storage, d_xp2)]
        idx_h = torch.empty(N0 * N1, dtype=torch.int32, pin_memory=True)
        res_h = torch.empty(2, dtype=torch.float64, pin_memory=True)
        cs = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        read = [torch.cuda.Event(), torch.cuda.Event()]

        def issue_copy(k):
            b = k % 2
            with torch.cuda.stream(cs):
                if k >= 2:
                    cs.wait_event(read[b])
                bufs[b][0][:nloc].copy_(xh, non_blocking=True)
                copied[b].record(cs)

        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        cs.wait_stream(torch.cuda.current_stream())
        issue_copy(0)
        for k in range(a.e2e_steps):
            if k + 1 < a.e2e_steps:
                issue_copy(k + 1)
            b = k % 2
            torch.cuda.current_stream().wait_event(copied[b])
            step(k, bufs[b][1], read[b])
            with torch.cuda.stream(side):  # the results of step k, after its finish
                res_h.copy_(sum_var, non_blocking=True)
                idx_h.copy_(idx.storage[:N0 * N1], non_blocking=True)
        join()
        f1.record()
        barrier()
        ems = f0.elapsed_time(f1) / a.e2e_steps
        te = torch.tensor([ems], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        ems = float(te.item())
        e2e = {"value": round(ntot / (ems * 1e-3) / 1e9, 4), "unit": "Gelem/s",
               "h2d_bytes_per_step": nloc * 4 * world, "d2h_bytes_per_step": (16 + N0 * N1 * 4) * world,
               "ms_per_step": round(ems, 3), "steps": a.e2e_steps,
               "overlap": "input copy of step k+1 under the kernels of step k (two input buffers)"}
        del x2, bufs, xh

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            cpu = cpu_baseline_single()
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "error": str(ex)[:200]}

    # ---- the other configurations' per-op reports (one GPU)
    per_config = None
    if world == 1 and not a.no_per_config:
        del x, y, z, xbufs, xp_view
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        per_config = per_config_block(peak)

    if rank == 0:
        value = ntot / (ms_max * 1e-3) / 1e9
        line = {
            "metric": "Gelem/s, strided-views step (permute->contiguous, x*0.5+exp(-x^2), sum/var, argmax axis 1)",
            "value": round(value, 4), "unit": "Gelem/s", "n_gpus": world, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": round(ms_max, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) from acd_rand (Philox4x32-10, seed 42, counter = "
            "global element index: identical for any GPU count)",
            "config": {"workload": "strided views 256x512x%d f32, sharded on axis 3" % n2,
                       "l2": "inputs larger than L2 (16 GiB), no flush needed",
                       "parallelism": "shard%d" % world, "elements": ntot},
            "roofline": {"bound": "hbm", "achieved": top["GB/s"], "peak": peak, "unit": "GB/s",
                         "frac": round(top["GB/s"] / peak, 4), "traffic": top["traffic"], "kernel": top["kernel"],
                         "peak_source": peak_kind, "traffic_source": "ncu dram bytes/elem of the 256x512x1024 "
                         "case x elements per launch",
                         "mix_ceiling": {"what": "acd_copy_fanout: the same bytes read once and written twice, "
                                         "contiguous streaming, this run", "GB/s": round(fan_gbs, 1),
                                         "frac": round(top["GB/s"] / fan_gbs, 4)}},
            "ops": ops,
            "phases_ms": phases,
            "gpu_launches": LAUNCHES_PER_STEP * a.steps,
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "result": {"sum": result_sum, "var": result_var, "argmax_axis1": result_idx},
            "per_config": per_config,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
