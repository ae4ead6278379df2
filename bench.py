#!/usr/bin/env python
"""Benchmark of the Fusion hot path on B200: the MLP training step through Fusion's
autodiff (4 Linear layers 1024-4096-4096-4096-16, ReLU, elementwise MSE, SGD
lr 1e-3, Kaiming-uniform init, global batch 65536), batch-sharded over N GPUs with an
NCCL all-reduce of the gradients.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line. `value` is whole-job samples/s with inputs already in HBM,
timed on the device with CUDA events over exactly K steps (max over ranks); `e2e`
is the same metric through the public API with the step's inputs copied from
pinned host memory and the loss read back every step. At N=1 the line also carries
the roofline of the dominant kernel (the 3xTF32 GEMM at the step's largest shape),
per-kernel bandwidth figures for the elementwise / reduction workloads, and the
reference CPU path timed on this host as a baseline.

`--impl reference` times the reference's own CPU implementation of the same step
(the Fusion C++ sources built into oracle/_ref) on a bounded sample of the batch.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
DIMS = [1024, 4096, 4096, 4096, 16]
GLOBAL_BATCH = 65536
LR = 1e-3
SEED = 1234
METRIC = ("MLP training step throughput (4x Linear 1024-4096-4096-4096-16 + ReLU, "
          "elementwise MSE, SGD lr 1e-3, fp32 with 3xTF32 GEMMs)")
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
REFERENCE_BUDGET_S = 240.0  # timed full-size reference steps stop once this has passed


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH, help="global batch")
    ap.add_argument("--no-kernels", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", default=None,
                    help="run one hot-path kernel on a profiling-sized case instead of the step "
                         "(step, gemm, gemm_full, gemm_wgrad, gemm_16384q, tf32_lo, add, bcast_add, exp, log, sqrt, sum_ax0, "
                         "sum_ax1, max_ax0, sum_rows64, swapaxes, bias_relu, linear_relu, gemm_epi_fwd, "
                         "gemm_epi_bwd)")
    ap.add_argument("--reps", type=int, default=3)
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "basis": "measured"}
    return dict(PEAKS_FALLBACK, basis="fallback")


def workload_config(batch, world):
    """The workload both arms report (the driver compares the two lines' configs)."""
    return {"workload": "mlp_train_step", "dims": DIMS, "global_batch": batch,
            "per_gpu_batch": batch // world, "parallelism": f"dp{world}", "lr": LR,
            "optimizer": "SGD momentum 0", "loss": "elementwise MSE (x/size)",
            "l2": "inputs and activations larger than L2 (1 GiB per [65536,4096] tensor)"}


def flops_per_sample():
    fwd = sum(2 * DIMS[i] * DIMS[i + 1] for i in range(len(DIMS) - 1))
    return 3 * fwd  # forward + input-grad and weight-grad GEMMs (layer-1 input grad included)


# ---------------------------------------------------------------- clocks
class Clocks:
    """Samples nvidia-smi during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.index)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------- distributed plumbing
class Dist:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def bcast_bytes(self, b):
        if not self.pg:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ---------------------------------------------------------------- device timing helpers
class Timer:
    def __init__(self, capi):
        self.A, self.L = capi, capi.lib()
        self.h = C.c_void_p()
        capi.check(self.L.fz_timer_create(C.byref(self.h)))

    def start(self):
        self.A.check(self.L.fz_timer_start(self.h, None))

    def stop_ms(self):
        self.A.check(self.L.fz_timer_stop(self.h, None))
        ms = C.c_float()
        self.A.check(self.L.fz_timer_elapsed_ms(self.h, C.byref(ms)))
        return float(ms.value)


def time_launch(capi, fn, reps=10, warm=3):
    t = Timer(capi)
    for _ in range(warm):
        fn()
    capi.check(capi.lib().fz_stream_sync(None))
    t.start()
    for _ in range(reps):
        fn()
    return t.stop_ms() / reps


def fused_program(capi, nodes, nleaves, outs):
    """An fz_program from (kind, op, src0, src1, imm) tuples (src < 0: leaf -1-src)."""
    p = capi.Program()
    p.num_nodes, p.num_leaves, p.num_outputs = len(nodes), nleaves, len(outs)
    for i, node in enumerate(outs):
        p.out_node[i] = node
    for i, (kind, op, s0, s1, imm) in enumerate(nodes):
        p.nodes[i].kind, p.nodes[i].op, p.nodes[i].src0, p.nodes[i].src1 = kind, op, s0, s1
        p.nodes[i].imm = imm
    return p


def kernel_suite(capi, pk):
    """Elementwise / reduction / GEMM workloads of the hot-path sweep, one line each."""
    L, A = capi.lib(), capi
    hbm = pk["hbm_gbs"]
    out = {}
    n = 1 << 28
    a, b, o = A.DeviceArray((n,)), A.DeviceArray((n,)), A.DeviceArray((n,))
    A.check(L.fz_fill_f32(a.ptr, C.c_float(0.5), n, None))
    A.check(L.fz_fill_f32(b.ptr, C.c_float(1.5), n, None))

    def rec(name, ms, nbytes):
        gbs = nbytes / ms / 1e6
        out[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 3)}

    for op in ("add", "mul", "div"):
        rec(f"{op}_2^28", time_launch(A, lambda: A.check(L.fz_ewise_binary_contig(
            A.BINOPS[op], n, o.ptr, a.ptr, b.ptr, None))), 12 * n)
    for e in (20, 22, 24, 25, 26, 27):  # the sweep's smaller sizes
        k = 1 << e
        rec(f"add_2^{e}", time_launch(A, lambda: A.check(L.fz_ewise_binary_contig(
            0, k, o.ptr, a.ptr, b.ptr, None))), 12 * k)
        if 12 * k <= 126 << 20:  # the three operands fit the 126 MB L2: an L2 rate, not HBM
            out[f"add_2^{e}"]["l2_resident"] = True
    plan = A.make_plan((n,), [(n,), (n,)])
    for op in ("exp", "log", "sqrt"):
        rec(f"{op}_2^28", time_launch(A, lambda: A.check(L.fz_ewise_unary(
            A.UNOPS[op], C.byref(plan), o.ptr, a.ptr, None))), 8 * n)
    r = 16384
    bplan = A.make_plan((r, r), [(r, r), (r, r), (1, r)])
    rec("bcast_add_16384^2+[1,16384]", time_launch(A, lambda: A.check(L.fz_ewise_binary(
        0, C.byref(bplan), o.ptr, a.ptr, b.ptr, None))), 8 * r * r + 4 * r)
    s = 8192
    for name, (outer, ln, inner) in (("sum_ax1_8192^2", (s, s, 1)), ("sum_ax0_8192^2", (1, s, s)),
                                     ("mean_ax1_8192^2", (s, s, 1)), ("mean_ax0_8192^2", (1, s, s)),
                                     ("max_ax1_8192^2", (s, s, 1)), ("max_ax0_8192^2", (1, s, s))):
        op = 2 if name.startswith("max") else 1 if name.startswith("mean") else 0
        rec(name, time_launch(A, lambda: A.check(L.fz_reduce(op, o.ptr, a.ptr, outer, ln, inner, None))),
            4 * s * s + 4 * (outer * inner))
    # [64,256,64,64] over (0,2,3), keepdims: the reference reduces one axis per call
    def chain4d():
        A.check(L.fz_reduce(0, o.ptr, a.ptr, 64 * 256 * 64, 64, 1, None))
        A.check(L.fz_reduce(0, b.ptr, o.ptr, 64 * 256, 64, 1, None))
        A.check(L.fz_reduce(0, o.ptr, b.ptr, 1, 64, 256, None))
    rec("sum_4d_axes023_chained", time_launch(A, chain4d), 4 * 64 * 256 * 64 * 64)
    # the same through the Python API: x.sum(3, True).sum(2, True).sum(0, True), where the
    # host joins the adjacent axes 2 and 3 into one pass (rows of 4096), then axis 0
    import nova_b200

    F = nova_b200.fusion
    dev = F.CppDevice(F.CppDeviceType.CPU, 0)
    x4 = np.random.default_rng(SEED + 3).standard_normal((64, 256, 64, 64), dtype=np.float32)
    t4 = F.Tensor(list(x4.shape), x4.ravel(), F.CppDType.FLOAT32, dev, False)
    del x4
    rec("sum_4d_axes023_api", time_launch(A, lambda: F.flush(t4.sum(3, True).sum(2, True).sum(0, True))),
        4 * 64 * 256 * 64 * 64)
    del t4
    shp = (C.c_int64 * 2)(r, r)
    rec("swapaxes_16384^2", time_launch(A, lambda: A.check(L.fz_swapaxes(o.ptr, a.ptr, shp, 2, 0, 1, None))),
        8 * r * r)
    # Backward formulas (the registry's, as the fusion IR lowers them: one fused program
    # per op, sibling gradients of a binary op as two outputs of one program), upstream
    # gradient g ~ U(-1,1), x ~ U(-1,1) (U(0.01,10) for log/sqrt), y ~ U(0.5,2); 2^28
    # elements; algorithmic bytes as counted for the backward sweep.
    rng = np.random.default_rng(SEED + 5)
    m = n
    def uni(lo, hi):
        return A.DeviceArray.from_numpy(rng.random(m, dtype=np.float32) * np.float32(hi - lo)
                                        + np.float32(lo))
    ga, xa, xp, ya = uni(-1, 1), uni(-1, 1), uni(0.01, 10), uni(0.5, 2)
    o2 = A.DeviceArray((m,))
    BI, UN, CO = A.NODE_BINARY, A.NODE_UNARY, A.NODE_CONST
    bo, uo = A.BINOPS, A.UNOPS
    # name: (nodes with leaf i referenced as -1-i, leaves, output nodes, bytes per element)
    progs = {
        "add_bwd_accumulate": ([(BI, bo["add"], -1, -2, 0.0)], [ga, xa], [0], 12),
        "sub_bwd": ([(CO, 0, 0, 0, 0.0), (BI, bo["sub"], 0, -1, 0.0)], [ga], [1], 8),
        "mul_bwd": ([(BI, bo["mul"], -1, -3, 0.0), (BI, bo["mul"], -1, -2, 0.0)], [ga, xa, ya],
                    [0, 1], 20),
        "div_bwd": ([(BI, bo["div"], -1, -3, 0.0), (CO, 0, 0, 0, 0.0), (BI, bo["sub"], 1, -1, 0.0),
                     (BI, bo["mul"], 2, -2, 0.0), (BI, bo["mul"], -3, -3, 0.0),
                     (BI, bo["div"], 3, 4, 0.0)], [ga, xa, ya], [0, 5], 20),
        "exp_bwd": ([(UN, uo["exp"], -2, 0, 0.0), (BI, bo["mul"], -1, 0, 0.0)], [ga, xa], [1], 12),
        "log_bwd": ([(BI, bo["div"], -1, -2, 0.0)], [ga, xp], [0], 12),
        "sqrt_bwd": ([(UN, uo["sqrt"], -2, 0, 0.0), (CO, 0, 0, 0, 2.0), (BI, bo["mul"], 0, 1, 0.0),
                      (BI, bo["div"], -1, 2, 0.0)], [ga, xp], [3], 12),
        "relu_bwd": ([(CO, 0, 0, 0, 0.0), (BI, bo["gt"], -2, 0, 0.0), (BI, bo["mul"], -1, 1, 0.0)],
                     [ga, xa], [2], 12),
    }
    for name, (nodes, leaf_arrays, outs, per_elem) in progs.items():
        prog = fused_program(A, nodes, len(leaf_arrays), outs)
        plan = A.make_plan((m,), [(m,)] * (len(outs) + len(leaf_arrays)))
        leaves = (C.c_void_p * len(leaf_arrays))(*[arr.ptr for arr in leaf_arrays])
        optrs = (C.c_void_p * len(outs))(*[arr.ptr for arr in (o, o2)[:len(outs)]])
        ms = time_launch(A, lambda: A.check(L.fz_fused_launch(C.byref(prog), C.byref(plan), optrs,
                                                               leaves, None)))
        rec(name + "_2^28", ms, per_elem * m)
    for arr in (a, b, o, o2, ga, xa, xp, ya):
        arr.free()
    # GEMM sweep (N(0,1)/sqrt(K) operands), whole fz_gemm_f32 call including the remainder
    # split: square M=N=K (A [M,K], B [K,N]), the transpose-B variant (B given [N,K]), the
    # batched [64,512,512]^2, the weight-gradient shape x^T @ g (K = 65536 batch rows, both
    # operands MN-major) and the linear+ReLU forward of [512,1024] x [1024,512] (+ bias, ReLU)
    gemms = [(f"gemm_3xtf32_{s}^3", (1, s, s, s, 0, 0)) for s in (1024, 2048, 4096, 8192, 16384)]
    gemms += [("gemm_3xtf32_8192^3_transB", (1, 8192, 8192, 8192, 0, 1)),
              ("gemm_3xtf32_batched_64x512^3", (64, 512, 512, 512, 0, 0)),
              ("gemm_3xtf32_wgrad_4096x4096x65536", (1, 4096, 4096, 65536, 1, 0))]
    for name, (bt, M, N, K, tA, tB) in gemms:
        x = _random_device(A, (bt, K, M) if tA else (bt, M, K), 21)
        y = _random_device(A, (bt, N, K) if tB else (bt, K, N), 22)
        c = A.DeviceArray((bt, M, N))
        lda, ldb = (M if tA else K), (K if tB else N)
        reps = 3 if M * N * K >= 16384 ** 3 else 5
        ms = time_launch(A, lambda: A.check(L.fz_gemm_f32(bt, M, N, K, x.ptr, lda, M * K, tA, y.ptr,
                                                          ldb, N * K, tB, c.ptr, N, M * N, None)),
                         reps=reps, warm=2)
        tf = 2.0 * bt * M * N * K / ms / 1e9
        out[name] = {"ms": round(ms, 3), "TFLOP/s": round(tf, 1), "tensor_pipe_TFLOP/s": round(3 * tf, 1),
                     "frac_of_3xtf32_ceiling": round(tf / (pk["bf16_tflops"] / 6.0), 3)}
        for arr in (x, y, c):
            arr.free()
    out["linear_relu_512x1024x512"] = linear_relu_case(capi)
    return out


def linear_relu_case(capi):
    """C = relu(A @ B + bias), A [512,1024], B [1024,512], bias [512], through the Python
    API (GEMM, then the fused bias+ReLU program): device time per call."""
    import nova_b200

    F = nova_b200.fusion
    rng = np.random.default_rng(SEED + 9)
    dev = F.CppDevice(F.CppDeviceType.CPU, 0)

    def t(a):
        return F.Tensor(list(a.shape), a.ravel(), F.CppDType.FLOAT32, dev, False)
    Am = t(rng.standard_normal((512, 1024), dtype=np.float32))
    Bm = t(rng.standard_normal((1024, 512), dtype=np.float32))
    bias = t(rng.uniform(-0.1, 0.1, 512).astype(np.float32))
    ms = time_launch(capi, lambda: F.flush((Am @ Bm + bias).maximum(0.0)), reps=20, warm=3)
    return {"ms": round(ms, 4), "TFLOP/s": round(2.0 * 512 * 1024 * 512 / ms / 1e9, 2)}


def _random_device(capi, shape, seed):
    a = np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
    return capi.DeviceArray.from_numpy(a)


def gemm_roofline(recs, pk, steps, step_ms):
    """Roofline of the step's dominant kernel from its launches inside the timed
    steps: each GEMM main-kernel launch was bracketed by a CUDA event pair on its own
    stream (fz_gemm_timing). Launches are grouped by product shape and schedule; the
    group with the most device time is the dominant kernel. Achieved = 2*batch*M*N*K
    per launch / its mean duration. The launches run inside a long, power-capped step,
    so the peak is the sustained measured bf16 rate / 2 (TF32) / 3 (3xTF32 issues three
    TF32 MMAs per product); the fraction of the burst rate is reported beside it."""
    groups = {}
    for r in recs:
        key = (r.batch, r.M, r.N, r.K, r.pair)
        g = groups.setdefault(key, {"ms": [], "epilogue": 0, "splits": r.splits})
        g["ms"].append(r.ms)
        g["epilogue"] += r.epilogue
    if not groups:
        return None
    (b, M, N, K, pair), g = max(groups.items(), key=lambda kv: sum(kv[1]["ms"]))
    ms = statistics.fmean(g["ms"])
    flops = 2.0 * b * M * N * K
    achieved = flops / ms / 1e9
    tf32_sust = pk["bf16_tflops_sustained"] / 2.0
    tf32_burst = pk["bf16_tflops"] / 2.0
    peak = tf32_sust / 3.0
    traffic = None
    summary = ROOT / "profiles" / "gemm_3xtf32_mlp_layer.md"
    if summary.exists():
        for line in summary.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch_full_size:"):
                traffic = float(line.split(":", 1)[1])
    total_gemm = sum(sum(v["ms"]) for v in groups.values())
    kname = "gemm_pair_kernel (cta_group::2)" if pair else "gemm_3xtf32_kernel"
    return {"kernel": f"{kname} 3xTF32, product [{M},{K}]x[{K},{N}]" + (f" x{b}" if b > 1 else ""),
            "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
            "unit": "TFLOP/s", "frac": round(achieved / peak, 3), "traffic": traffic,
            "peak_basis": (f"{pk['basis']} sustained bf16 {pk['bf16_tflops_sustained']} TFLOP/s "
                           f"/ 2 (TF32 rate) / 3 (3xTF32): the launches are timed inside the step"),
            "frac_of_burst": round(achieved / (tf32_burst / 3.0), 3),
            "tensor_pipe_achieved": round(3 * achieved, 1),
            "launches_timed": len(g["ms"]), "launches_per_step": round(len(g["ms"]) / steps, 2),
            "with_fused_epilogue": g["epilogue"], "k_splits": g["splits"],
            "ms_per_launch": round(ms, 3), "ms_per_launch_min": round(min(g["ms"]), 3),
            "ms_per_launch_max": round(max(g["ms"]), 3),
            "share_of_step": round(sum(g["ms"]) / steps / step_ms, 3),
            "all_gemms_share_of_step": round(total_gemm / steps / step_ms, 3),
            "timing": "CUDA events around each launch on the launching stream, inside the timed steps",
            "algorithmic_bytes_per_launch": 4.0 * b * (2 * M * K + 2 * N * K + M * N)}


def cpu_baseline_ref(batch=4096, steps=1):
    """The reference CPU path (oracle/_ref: Fusion's C++ sources + OpenBLAS) on a bounded
    sample of the workload: `steps` MLP steps on `batch` rows after one warm-up step,
    wall clock (about 30 s on the host). A reference step's cost has a part fixed per
    step (transposes of the 4096x4096 weights) and a part per row, so this sample
    understates the full batch's rate a little; `bench.py --impl reference` times the
    full batch."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    from nova_b200.mlp import init_params

    R = oracle.Ref()
    rng = np.random.default_rng(SEED + 7)
    X = rng.standard_normal((batch, DIMS[0])).astype(np.float32)
    Y = rng.standard_normal((batch, DIMS[-1])).astype(np.float32)
    Ws, bs = init_params(DIMS, SEED)
    Ws, bs, _ = R.mlp_step(X, Y, Ws, bs, LR)  # warm-up
    t0 = time.perf_counter()
    for _ in range(steps):
        Ws, bs, _ = R.mlp_step(X, Y, Ws, bs, LR)
    dt = (time.perf_counter() - t0) / steps
    return {"value": round(batch / dt, 2), "unit": "samples/s", "cores": os.cpu_count(),
            "kind": "reference",
            "sample": f"{steps} steps of the same MLP step on {batch} rows (reference Fusion C++ "
                      f"autodiff + OpenBLAS sgemm with all host threads; elementwise ops "
                      f"single-threaded as in the reference), {dt * 1e3:.0f} ms/step"}


# ---------------------------------------------------------------- our arm
def run_ours(args):
    # NCCL writes its log (with NCCL_DEBUG set, a version banner at least) to stdout, where
    # the one JSON line goes: send it to stderr unless a log file was chosen
    if os.environ.get("NCCL_DEBUG") and not os.environ.get("NCCL_DEBUG_FILE"):
        os.environ["NCCL_DEBUG_FILE"] = "/dev/stderr"
    d = Dist()
    import nova_b200
    from nova_b200 import capi
    from nova_b200.mlp import MLP, init_params

    F = nova_b200.fusion
    F.set_device(d.local)
    comm = None
    if d.world > 1:
        uid = d.bcast_bytes(F.comm_unique_id() if d.rank == 0 else None)
        comm = F.Comm(d.world, d.rank, uid)
    assert args.batch % d.world == 0, "global batch must divide by the number of GPUs"
    local = args.batch // d.world
    Ws, bs = init_params(DIMS, SEED)
    model = MLP(F, Ws, bs)
    rng = np.random.default_rng(SEED + 1 + d.rank)
    Xh = rng.standard_normal((local, DIMS[0]), dtype=np.float32)
    Yh = rng.standard_normal((local, DIMS[-1]), dtype=np.float32)
    # pinned host copies for the end-to-end leg
    L = capi.lib()
    pin = []
    for src in (Xh, Yh):
        p = C.c_void_p()
        capi.check(L.fz_host_alloc(C.byref(p), src.nbytes))
        arr = np.ctypeslib.as_array((C.c_float * src.size).from_address(p.value)).reshape(src.shape)
        arr[...] = src
        pin.append((p, arr))
    Xp, Yp = pin[0][1], pin[1][1]
    X = model.tensor(Xh, True)  # nova's Tensor defaults to requires_grad=True
    Y = model.tensor(Yh, True)

    kernels = None
    if d.world == 1 and not args.no_kernels:
        # per-kernel sweep first, on a GPU not yet heated by the GEMM-bound step
        kernels = kernel_suite(capi, peaks())
    for _ in range(args.warmup):
        model.step(X, Y, LR, comm)
    F.synchronize()

    clocks = Clocks(d.local)
    timer = Timer(capi)
    clocks.start()  # sampling every 50 ms from the last warm-up step through the timed region
    model.step(X, Y, LR, comm)
    d.barrier()
    F.synchronize()
    launches0 = L.fz_launch_count()
    roofline_timing = d.world == 1 and d.rank == 0
    if roofline_timing:  # event pairs around each GEMM launch (the N=1 line's roofline)
        capi.check(L.fz_gemm_timing(1))
    timer.start()
    for _ in range(args.steps):
        loss = model.step(X, Y, LR, comm)
    ms_local = timer.stop_ms()
    F.synchronize()
    if comm:
        comm.wait(120.0)
    launches = L.fz_launch_count() - launches0
    gemm_recs = capi.gemm_timing_read() if roofline_timing else []
    capi.check(L.fz_gemm_timing(0))
    d.barrier()
    ms = d.max(ms_local) / args.steps

    clk = clocks.stop()  # sampled over the device-timed steps (the e2e leg syncs every step)

    # end to end: each step's inputs copied from pinned host memory and its loss mean read
    # back, pipelined as a training loop does: step i+1's inputs are uploaded (on the
    # upload stream) and its kernels submitted before step i's loss is read, so the copy
    # and the submission overlap step i on the GPU
    h2d = Xp.nbytes + Yp.nbytes

    def e2e_loop(n):
        pending = model.step(model.tensor(Xp, True), model.tensor(Yp, True), LR, comm).mean()
        F.flush(pending)  # the loss mean is launched right behind its step
        for i in range(n):
            nxt = None
            if i + 1 < n:
                nxt = model.step(model.tensor(Xp, True), model.tensor(Yp, True), LR, comm).mean()
                F.flush(nxt)
            pending.to_numpy()  # read back beside the next step
            pending = nxt

    # untimed warm-up of the same pipelined loop: compiles the read-back program and
    # lets the allocator set up the rotating upload buffers (a pool that grows inside
    # the timed steps stalls the host in the driver's allocation call)
    e2e_loop(max(3, args.warmup))
    d.barrier()
    F.synchronize()
    timer.start()
    e2e_loop(args.steps)
    F.synchronize()
    e2e_local = timer.stop_ms()
    F.synchronize()
    d.barrier()
    e2e_ms = d.max(e2e_local) / args.steps

    value = args.batch / (ms / 1e3)
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "samples/s", "n_gpus": d.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs/targets, Kaiming-uniform weights, zero biases)",
        "config": workload_config(args.batch, d.world),
        "e2e": {"value": round(args.batch / (e2e_ms / 1e3), 1), "unit": "samples/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4,
                "path": "nova_b200.fusion Python API (Tensor from pinned host arrays, "
                        "loss.mean().to_numpy(); next step submitted before the read)"},
        "gpu_launches": int(launches),
        "gpu_launches_per_step": round(launches / args.steps, 1),
        "model_tflops_per_step": round(flops_per_sample() * args.batch / 1e12, 2),
        "clocks": clk,
    }
    if d.world == 1 and d.rank == 0:
        pk = peaks()
        res["roofline"] = gemm_roofline(gemm_recs, pk, args.steps, ms)
        if kernels is not None:
            res["kernels"] = kernels
        if not args.no_cpu_baseline:
            try:
                res["cpu_baseline"] = cpu_baseline_ref()
            except Exception as e:  # oracle not built on this host
                res["cpu_baseline"] = {"value": None, "unavailable": str(e)}
    if comm:
        comm.destroy()
    for p, _ in pin:
        L.fz_host_free(p)
    if d.rank == 0:
        print(json.dumps(res), flush=True)
    d.close()


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's own CPU implementation of the step (Fusion's C++ sources and
    autodiff engine with OpenBLAS, built into oracle/_ref) on the full global batch.
    A step at 65536 rows costs minutes on the host (serial transposes of 1 GiB
    activations dominate), and the first one about twice the next (the reference's
    pool allocator grows), so: one full-size warm-up step, then full-size timed steps
    until `--steps` are done or the next would end after REFERENCE_BUDGET_S (at least one);
    `steps` reports the steps timed and `steps_requested` the flag."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    from nova_b200.mlp import init_params

    if not oracle.have_ref():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libfusion_ref.so not built (make -C oracle ref)"}))
        return
    R = oracle.Ref()
    rows = args.batch
    rng = np.random.default_rng(SEED + 1)
    X = rng.standard_normal((rows, DIMS[0]), dtype=np.float32)
    Y = rng.standard_normal((rows, DIMS[-1]), dtype=np.float32)
    Ws, bs = init_params(DIMS, SEED)
    t0 = time.perf_counter()
    Ws, bs, _ = R.mlp_step(X, Y, Ws, bs, LR)  # one full-size warm-up step
    warm = 1
    warm_s = time.perf_counter() - t0
    done = 0
    t0 = time.perf_counter()
    while done < args.steps:
        Ws, bs, _ = R.mlp_step(X, Y, Ws, bs, LR)
        done += 1
        spent = time.perf_counter() - t0
        if spent + spent / done > REFERENCE_BUDGET_S:  # the next step would overrun
            break
    dt = (time.perf_counter() - t0) / done
    v = round(rows / dt, 2)
    cores = os.cpu_count()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "samples/s",
        "n_gpus": world, "steps": done, "steps_requested": args.steps, "warmup": warm,
        "warmup_requested": args.warmup, "ms_per_step": round(dt * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs/targets, Kaiming-uniform weights, zero biases)",
        "config": workload_config(rows, world),
        "execution": (f"reference Fusion CPU path in one process on the host ({cores} threads for "
                      f"OpenBLAS sgemm; its elementwise ops, reductions and transposes are "
                      f"single-threaded); every step runs all {rows} rows; the GPUs are unused; "
                      f"warm-up step {warm_s:.0f} s"),
        "cpu_baseline": {"value": v, "unit": "samples/s", "cores": cores, "kind": "reference",
                         "sample": f"{done} full step(s) of {rows} rows after one warm-up step"},
        "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_kernel(args):
    """One kernel in a loop, sized for an ncu capture (inputs above L2, a few GB)."""
    import nova_b200
    from nova_b200 import capi

    F = nova_b200.fusion
    F.set_device(0)
    A, L = capi, capi.lib()
    k = args.kernel
    if k in ("gemm", "gemm_full", "gemm_wgrad", "gemm_16384q"):
        # gemm: the MLP's dominant forward shape x @ W^T at 1/8 of the batch (both operands
        # K-major); gemm_full: the same at the full 65536 rows (the roofline's product);
        # gemm_wgrad: the weight gradient x^T @ g at 1/4 of the batch (both MN-major).
        # Remainder planes split beforehand: the loop is the GEMM kernel alone.
        # gemm_16384q: the 16384^3 sweep product at a quarter of its rows (A [4096,16384],
        # B [16384,16384] read MN-major as in the sweep).
        m, n, kk, tA, tB = {"gemm": (8192, 4096, 4096, 0, 1), "gemm_full": (65536, 4096, 4096, 0, 1),
                            "gemm_wgrad": (4096, 4096, 16384, 1, 0),
                            "gemm_16384q": (4096, 16384, 16384, 0, 0)}[k]
        ash, bsh = ((kk, m) if tA else (m, kk)), ((n, kk) if tB else (kk, n))
        x, w, c = _random_device(A, ash, 1), _random_device(A, bsh, 2), A.DeviceArray((m, n))
        xl, wl = A.DeviceArray(ash), A.DeviceArray(bsh)
        A.check(L.fz_tf32_lo(xl.ptr, x.ptr, m * kk, None))
        A.check(L.fz_tf32_lo(wl.ptr, w.ptr, n * kk, None))
        fn = lambda: A.check(L.fz_gemm_f32_split(1, m, n, kk, x.ptr, xl.ptr, ash[1], 0, tA, w.ptr,
                                                  wl.ptr, bsh[1], 0, tB, c.ptr, n, 0, None))
        work = 2.0 * m * n * kk
    elif k in ("gemm_epi_fwd", "gemm_epi_bwd"):
        # the "gemm" product with the MLP's fused epilogues: forward relu(P + b) with its
        # remainder plane, backward P * (Y > 0) with its plane (Y the forward's ReLU output)
        m, n, kk = 8192, 4096, 4096
        x, w = _random_device(A, (m, kk), 1), _random_device(A, (n, kk), 2)
        xl, wl = A.DeviceArray((m, kk)), A.DeviceArray((n, kk))
        A.check(L.fz_tf32_lo(xl.ptr, x.ptr, m * kk, None))
        A.check(L.fz_tf32_lo(wl.ptr, w.ptr, n * kk, None))
        Bn, Un, Kn = A.NODE_BINARY, A.NODE_UNARY, A.NODE_CONST
        bo, uo = A.BINOPS, A.UNOPS
        bias, full = _random_device(A, (n,), 3), _random_device(A, (m, n), 4)
        if k == "gemm_epi_fwd":
            prog = fused_program(A, [(Bn, bo["add"], -1, -2, 0.0), (Kn, 0, 0, 0, 0.0),
                                     (Bn, bo["maximum"], 0, 1, 0.0), (Un, uo["tf32_lo"], 2, 0, 0.0)],
                                 2, [2, 3])
            ins = (A.EpiInput * 1)(A.EpiInput(bias.ptr, 0, 0, 1))
        else:
            prog = fused_program(A, [(Kn, 0, 0, 0, 0.0), (Bn, bo["gt"], -2, 0, 0.0),
                                     (Bn, bo["mul"], -1, 1, 0.0), (Un, uo["tf32_lo"], 2, 0, 0.0)],
                                 2, [2, 3])
            ins = (A.EpiInput * 1)(A.EpiInput(full.ptr, 0, n, 1))
        outs = [A.DeviceArray((m, n)) for _ in range(prog.num_outputs)]
        optr = (C.c_void_p * len(outs))(*[o.ptr for o in outs])
        fn = lambda: A.check(L.fz_gemm_f32_epilogue(1, m, n, kk, x.ptr, xl.ptr, kk, 0, 0, w.ptr, wl.ptr,
                                                     kk, 0, 1, C.byref(prog), ins, optr, n, 0, None))
        work = 2.0 * m * n * kk
    elif k == "step":  # the MLP training step alone (reps steps), for a launch list
        from nova_b200.mlp import MLP, init_params

        Ws, bs = init_params(DIMS, SEED)
        model = MLP(F, Ws, bs)
        rng = np.random.default_rng(SEED + 1)
        X = model.tensor(rng.standard_normal((args.batch, DIMS[0]), dtype=np.float32), True)
        Y = model.tensor(rng.standard_normal((args.batch, DIMS[-1]), dtype=np.float32), True)

        def fn():
            model.step(X, Y, LR)
        work = float(args.batch)
    elif k == "tf32_lo":  # remainder plane of a [65536,4096] activation (GEMM operand split)
        n = 1 << 28
        a, o = _random_device(A, (n,), 3), A.DeviceArray((n,))
        fn = lambda: A.check(L.fz_tf32_lo(o.ptr, a.ptr, n, None))
        work = 8.0 * n
    elif k == "linear_relu":  # relu(x @ W^T + b) through the API: the GEMM with its epilogue
        rows, cols, kk = 8192, 4096, 4096
        rng = np.random.default_rng(SEED + 5)
        dev = F.CppDevice(F.CppDeviceType.CPU, 0)
        mk = lambda shp: F.Tensor(list(shp), rng.standard_normal(shp, dtype=np.float32).ravel(),
                                  F.CppDType.FLOAT32, dev, False)
        xt, wt, bt = mk((rows, kk)), mk((cols, kk)), mk((cols,))
        wT = wt.swapaxes(1, 0)
        F.flush(wT)

        def fn():
            F.flush((xt @ wT + bt).maximum(0.0))
        work = 2.0 * rows * cols * kk
    elif k == "bias_relu":  # fused relu(x + b) of the MLP forward through the fusion IR
        rows, cols = 16384, 4096
        dev = F.CppDevice(F.CppDeviceType.CPU, 0)
        xt = F.Tensor([rows, cols], np.zeros(rows * cols, np.float32), F.CppDType.FLOAT32, dev, False)
        bt = F.Tensor([cols], np.zeros(cols, np.float32), F.CppDType.FLOAT32, dev, False)

        def fn():
            F.flush((xt + bt).maximum(0.0))
        work = 8.0 * rows * cols
    else:
        n = 1 << 26
        a, b, o = A.DeviceArray((n,)), A.DeviceArray((n,)), A.DeviceArray((n,))
        A.check(L.fz_fill_f32(a.ptr, C.c_float(0.5), n, None))
        A.check(L.fz_fill_f32(b.ptr, C.c_float(1.5), n, None))
        r = 8192
        plan1 = A.make_plan((n,), [(n,), (n,)])
        bplan = A.make_plan((r, r), [(r, r), (r, r), (1, r)])
        shp = (C.c_int64 * 2)(r, r)
        q = 1 << 20  # [64,256,64,64] as 2^20 rows of 64 (first call of the axes-(0,2,3) chain)
        fn, work = {
            "add": (lambda: A.check(L.fz_ewise_binary_contig(0, n, o.ptr, a.ptr, b.ptr, None)), 12.0 * n),
            "exp": (lambda: A.check(L.fz_ewise_unary(0, C.byref(plan1), o.ptr, a.ptr, None)), 8.0 * n),
            "log": (lambda: A.check(L.fz_ewise_unary(1, C.byref(plan1), o.ptr, a.ptr, None)), 8.0 * n),
            "sqrt": (lambda: A.check(L.fz_ewise_unary(2, C.byref(plan1), o.ptr, a.ptr, None)), 8.0 * n),
            "max_ax0": (lambda: A.check(L.fz_reduce(2, o.ptr, a.ptr, 1, r, r, None)), 4.0 * r * r),
            "sum_rows64": (lambda: A.check(L.fz_reduce(0, o.ptr, a.ptr, q, 64, 1, None)), 4.0 * q * 64),
            "bcast_add": (lambda: A.check(L.fz_ewise_binary(0, C.byref(bplan), o.ptr, a.ptr, b.ptr, None)),
                          8.0 * r * r + 4 * r),
            "sum_ax1": (lambda: A.check(L.fz_reduce(0, o.ptr, a.ptr, r, r, 1, None)), 4.0 * r * r),
            "sum_ax0": (lambda: A.check(L.fz_reduce(0, o.ptr, a.ptr, 1, r, r, None)), 4.0 * r * r),
            "swapaxes": (lambda: A.check(L.fz_swapaxes(o.ptr, a.ptr, shp, 2, 0, 1, None)), 8.0 * r * r),
        }[k]
    ms = time_launch(A, fn, reps=args.reps, warm=1)
    F.synchronize()
    gemm = k.startswith("gemm") or k == "linear_relu"
    unit = "TFLOP/s" if gemm else "samples/s" if k == "step" else "GB/s"
    scale = 1e9 if gemm else 1e-3 if k == "step" else 1e6
    print(json.dumps({"kernel": k, "ms": round(ms, 4), unit: round(work / ms / scale, 1)}),
          flush=True)


def main():
    args = parse()
    if args.kernel:
        run_kernel(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
