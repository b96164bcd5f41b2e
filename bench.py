"""Benchmark of sumac_b200 on BASELINE.json's metric.

Workload (default): config C4, the graph-shaped square matrix m = n = 139255 with 19,773,733
nonzeros (log-normal degrees, endpoints proportional to degree, values log(1+k), k geometric),
factorised by SALSA with rank 16 and 100 blocks. The data are seeded synthetic stand-ins for the
connectome matrix (the real dataset is not available here).

One step = one SALSA iteration (two reshuffles, CSR rebuilds and 2 x 100 block updates) with the
data already resident on the GPU. `value` = iterations/s of the whole job (max over ranks).
`e2e` = the same metric through sumac_factorize() with the inputs in host memory (copies, pruning,
initialisation and validation included). The fused tcgen05 product of one block update is also
timed alone with CUDA events for the roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c4|c3|c2]
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (generator, rank, num_blocks, description)
    "c4": dict(rank=16, num_blocks=100, desc="C4 graph-shaped 139255x139255, nnz 19773733, SALSA rank 16, 100 blocks"),
    "c3": dict(rank=64, num_blocks=50, desc="C3 bigram-shaped 50000x50000, nnz~10M, SALSA rank 64, 50 blocks"),
    "c2": dict(rank=32, num_blocks=20, desc="C2 digits-shaped 70000x784, density 0.19, SALSA rank 32, 20 blocks"),
    "c5": dict(rank=64, num_blocks=123, desc="C5 power-law 1000000x1000000, nnz 2e8, GD rank 64, "
               "8131-row blocks (minibatch 8192), Adam", method="GD"),
}


# ------------------------------------------------------------------------------ synthetic data
def _sample_pairs(rng, p_row, p_col, n_cols, target):
    """Distinct (row, col) pairs drawn with probability p_row[r] p_col[c] (inverse-CDF sampling,
    duplicates merged, topped up until `target` distinct pairs, then a uniform subset). The
    uniforms come from the seeded numpy generator; the integer work runs in torch (on the GPU when
    there is one), so the result does not depend on where it runs."""
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cr = torch.from_numpy(np.cumsum(p_row)).to(dev)
    cc = torch.from_numpy(np.cumsum(p_col)).to(dev)
    cr /= cr[-1].clone()
    cc /= cc[-1].clone()
    keys = torch.empty(0, dtype=torch.int64, device=dev)
    while keys.numel() < target:
        need = int((target - keys.numel()) * 1.3) + 10000
        u = torch.from_numpy(rng.random(need)).to(dev)
        r = torch.clamp(torch.searchsorted(cr, u), max=p_row.size - 1)
        u = torch.from_numpy(rng.random(need)).to(dev)
        c = torch.clamp(torch.searchsorted(cc, u), max=p_col.size - 1)
        keys = torch.unique(torch.cat([keys, r * n_cols + c]))
    keys = keys.cpu().numpy()
    if keys.size > target:
        keys = np.sort(keys[rng.permutation(keys.size)[:target]])
    return keys


def make_c1(seed=0, m=2000, n=1500, d=8):
    """C1, the planted problem: A*, B* with N(0, sigma^2) entries, sigma^2 = 1/sqrt(8) (density
    ~29 %, the reading of "~25 %" that matches), S = ReLU(A* B*^T + N(0, 0.05^2) - 0.5), positives
    as COO. The product is accumulated term by term in float64 with separate multiplies and adds,
    so the data are the same on every machine (no BLAS summation order involved)."""
    rng = np.random.default_rng(seed)
    sigma = 8.0 ** -0.25
    A = rng.standard_normal((m, d)) * sigma
    B = rng.standard_normal((n, d)) * sigma
    L = np.zeros((m, n))
    for k in range(d):
        L = L + np.multiply.outer(A[:, k], B[:, k])
    L = L + 0.05 * rng.standard_normal((m, n)) - 0.5
    S = np.maximum(L, 0.0).astype(np.float32)
    rows, cols = np.nonzero(S)
    return np.stack([rows, cols]).astype(np.int64), S[rows, cols], (m, n)


def make_c4(seed=4, m=139255, nnz=19773733):
    rng = np.random.default_rng(seed)
    deg_out = rng.lognormal(4.2, 1.3, m)
    deg_in = rng.lognormal(4.2, 1.3, m)
    keys = _sample_pairs(rng, deg_out / deg_out.sum(), deg_in / deg_in.sum(), m, nnz)
    k = rng.geometric(0.3, nnz)
    vals = np.log1p(k).astype(np.float32)
    return np.stack([keys // m, keys % m]), vals, (m, m)


def make_c3(seed=3, m=50000, nnz=10_000_000):
    rng = np.random.default_rng(seed)
    w = 1.0 / np.arange(1, m + 1) ** 1.1
    pr = rng.permutation(w) / w.sum()
    pc = rng.permutation(w) / w.sum()
    keys = _sample_pairs(rng, pr, pc, m, nnz)
    c = rng.zipf(2.0, nnz)
    return np.stack([keys // m, keys % m]), np.log1p(c).astype(np.float32), (m, m)


def make_c2(seed=2, m=70000, n=784, density=0.19):
    rng = np.random.default_rng(seed)
    lo, hi = int(0.2 * n), int(0.8 * n)
    nnz = int(density * m * n)
    keys = np.sort(rng.choice(m * (hi - lo), nnz, replace=False))
    rows, cols = keys // (hi - lo), keys % (hi - lo) + lo
    big = rng.random(nnz) < 0.4
    vals = np.where(big, rng.uniform(0.9, 1.0, nnz), rng.uniform(0.0, 0.9, nnz))
    vals = np.maximum(vals, 1e-3).astype(np.float32)
    return np.stack([rows, cols]), vals, (m, n)


def make_c5(seed=5, m=1_000_000, nnz=200_000_000):
    """C5: C4's degree and value distributions at m = n = 10^6, nnz = 2 x 10^8."""
    return make_c4(seed=seed, m=m, nnz=nnz)


MAKERS = {"c1": make_c1, "c4": make_c4, "c3": make_c3, "c2": make_c2, "c5": make_c5}


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------ helpers
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def measure_tf32_matmul(device):
    """Dense TF32 throughput of torch.matmul (cuBLAS) on this GPU, 8192^3, best of 5."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device=device)
    b = torch.randn(8192, 8192, device=device)
    for _ in range(3):
        a @ b
    best = float("inf")
    for _ in range(5):
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        a @ b
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def tf32_round(t):
    """fp32 values rounded to the nearest tf32 value (ties to even), as the library packs F."""
    u = t.contiguous().view(torch.int32)
    u = (u + 0xFFF + ((u >> 13) & 1)) & -8192
    return u.view(torch.float32)


def dist_info():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ------------------------------------------------------------------------------ our arm
def run_ours(args):
    from sumac_b200 import SumacConfig, SumacMethod, _native, ops, sumac_factorize
    from sumac_b200.data import prune_zero_rows_cols
    from sumac_b200.salsa import SalsaState, draw_perm, init_salsa_factors

    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    cfgd = CONFIGS[args.config]
    idx_np, val_np, shape = MAKERS[args.config]()
    idx_h = torch.from_numpy(idx_np)
    val_h = torch.from_numpy(val_np)
    d, nb = cfgd["rank"], cfgd["num_blocks"]
    allow_tf32 = args.precision == "tf32"

    # ---- device-resident timed region (value)
    S_index = idx_h.to(dev)
    S_value = val_h.to(dev)
    S_index, _, _, m, n = prune_zero_rows_cols(S_index, shape)
    cfg = SumacConfig(method=SumacMethod.SALSA, rank=d, num_blocks=nb, seed=0, verbose=False,
                      allow_tf32=allow_tf32, device=dev)
    gen, gen_rows, gen_cols = cfg.get_generator()
    A, B = init_salsa_factors(S_index, S_value, m, n, d, gen)
    if world > 1:
        # rows of A and B sharded over the ranks (NCCL), total work fixed: strong scaling
        from sumac_b200.shard import ShardedSalsaState
        st = ShardedSalsaState(S_index, S_value, m, n, cfg, A, B)
    else:
        st = SalsaState(S_index, S_value, m, n, cfg, A, B)
    for it in range(1, args.warmup + 1):
        st.iteration(it, draw_perm(m, gen_rows, dev), draw_perm(n, gen_cols, dev))
    torch.cuda.synchronize()
    _native.raise_device_error(dev)
    if world > 1:
        dist.barrier()
    lib = _native.lib()
    launches0 = lib.sumac_kernel_launches() + st.replayed_launches
    ev0, ev1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with ClockSampler(local) as clk:
        ev0.record()
        for it in range(args.warmup + 1, args.warmup + args.steps + 1):
            st.iteration(it, draw_perm(m, gen_rows, dev), draw_perm(n, gen_cols, dev))
        ev1.record()
        torch.cuda.synchronize()
    # graph replays launch the kernels captured once: the library counts launches at capture
    launches = lib.sumac_kernel_launches() + st.replayed_launches - launches0
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    _native.raise_device_error(dev)
    ms_per_step = ms / args.steps
    value = args.steps / (ms * 1e-3)  # whole-job iterations/s (every rank runs every iteration)

    # ---- the fused product alone (one B-update of this rank's rows), CUDA events
    prec = cfg.precision()
    Dp = ops.padded_rank(d)
    b = (m + nb - 1) // nb
    n_loc = st.Bp.shape[0]  # this rank's rows of B (all of them on one GPU)
    rows = torch.randperm(st.Ap.shape[0], device=dev)[:b]
    FI = st.Ap[rows].contiguous()
    x3 = prec == ops.SUMAC_3XTF32
    ldct = (b + 3) // 4 * 4
    Ct = torch.zeros((Dp, ldct), device=dev)
    Ct[:, :b] = torch.randn(b, Dp, device=dev).T * 1e-2
    if x3:
        Fhi = (FI.view(torch.int32) & -8192).view(torch.float32)
        Flo = FI - Fhi
        Cthi = (Ct.view(torch.int32) & -8192).view(torch.float32)
        Ctlo = Ct - Cthi
    else:
        Fhi, Flo, Cthi, Ctlo = tf32_round(FI), None, Ct, None
    splits = lib.sumac_relu_product_splits(n_loc, b, Dp, prec)
    part = torch.empty(splits * n_loc * Dp + 16, device=dev)
    err = _native.err_word(dev)
    stream = _native.stream_ptr(dev)
    P = _native.ptr

    def launch():
        _native.check(lib.sumac_relu_product(P(st.Bp), n_loc, P(Fhi), P(Flo), P(Cthi), P(Ctlo), ldct,
                                             b, Dp, prec, P(part), P(err), stream), "relu_product")
    for _ in range(5):
        launch()
    reps = 50
    k0, k1 = torch.cuda.Event(True), torch.cuda.Event(True)
    k0.record()
    for _ in range(reps):
        launch()
    k1.record()
    torch.cuda.synchronize()
    _native.raise_device_error(dev)
    kernel_ms = k0.elapsed_time(k1) / reps
    flops = 4.0 * n_loc * b * d
    achieved = flops / (kernel_ms * 1e-3) / 1e12
    pk = peaks()
    tf32_peak = pk["bf16_tflops"] / 2.0
    tf32_measured = measure_tf32_matmul(dev) if rank == 0 else None
    reduce_line = measure_reduce(dev, prec, tf32_peak) if rank == 0 else None

    # ---- e2e through the public API with host inputs
    e2e = None
    if not args.no_e2e:
        # every rank calls the public API (sharded over the process group when world > 1)
        cfg2 = SumacConfig(method=SumacMethod.SALSA, rank=d, num_blocks=nb, seed=0, verbose=False,
                           allow_tf32=allow_tf32, max_iterations=args.steps,
                           eval_interval=args.steps + 1, device=dev)
        idx_pin = idx_h.pin_memory()
        val_pin = val_h.pin_memory()
        # one untimed call of the same API first (warm-up: the process's first call pays one-time
        # library and allocator setup that varies by ~0.3 s between runs)
        cfg_w = dataclasses.replace(cfg2, max_iterations=max(1, args.warmup))
        sumac_factorize(S_index=idx_pin, S_value=val_pin, shape=shape, config=cfg_w)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        A2, B2, _ = sumac_factorize(S_index=idx_pin, S_value=val_pin, shape=shape, config=cfg2)
        torch.cuda.synchronize()
        t_e2e = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([t_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        h2d = idx_h.numel() * idx_h.element_size() + val_h.numel() * 4
        d2h = (A2.numel() + B2.numel()) * 4
        e2e = {"value": args.steps / t_e2e, "unit": "iter/s",
               "h2d_bytes_per_step": h2d / args.steps, "d2h_bytes_per_step": d2h / args.steps,
               "seconds": t_e2e, "note": "one sumac_factorize call of `steps` iterations with host "
               "inputs: copies, validation, pruning, init and CSR setup inside the timed region"}

    if rank != 0:
        _teardown(st, world)
        return
    cpu = cpu_baseline(args, idx_np, val_np, shape, d, nb) if not args.no_cpu else None
    clocks = clk.summary()
    line = {
        "metric": "fused ReLU(AB^T)-reduce TFLOP/s; GD/SALSA iters/s at 1/2/4/8 B200",
        "value": value, "unit": "iter/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "tf32" if not x3 else "f32 (3xTF32)", "data": "synthetic (seeded stand-in)",
        "config": bench_config(cfgd, m, n, val_np.size, world, args),
        "fused_product": {"tflops": achieved, "ms_per_launch": kernel_ms, "M": n_loc, "N": b, "d": d,
                          "splits": splits, "flops_per_launch": flops},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s",
                     "frac": achieved / tf32_peak,
                     # dram__bytes_read.sum + dram__bytes_write.sum of one launch at this shape
                     # (d = 16, TF32), ncu --set full: profiles/relu_product_c4_d16_tf32.md
                     "traffic": 9.14e6 if (d == 16 and not x3 and args.config == "c4") else None,
                     "peak_source": f"{pk['source']} bf16 / 2 (dense TF32 rate)",
                     "tf32_matmul_measured_tflops": tf32_measured},
        "fused_reduce": reduce_line,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "clocks": clocks,
        "gpu_launches": int(launches),
    }
    print(json.dumps(line), flush=True)
    _teardown(st, world)


def measure_reduce(dev, prec, tf32_peak):
    """relu_bat_reduce (sum ReLU(A B^T), sum ReLU(A B^T)^2) at the reference's benchmark shapes
    (kernel_benchmarks/relu_bat_reduce_bench.py:193-202: M=288768, N=1408, D in 16..256), flops
    M N (2D-1) + 3 M N (:19-24), CUDA events over 20 launches of the C entry point."""
    from sumac_b200 import _native
    lib = _native.lib()
    M, Nr = 288768, 1408
    g = torch.Generator(device=dev).manual_seed(1)
    P = _native.ptr
    err = _native.err_word(dev)
    stream = _native.stream_ptr(dev)
    res = {"M": M, "N": Nr, "note": "operands L2-resident (the kernel is tensor / issue bound)"}
    for D in (16, 32, 64, 128, 256):
        A = torch.randn(M, D, device=dev, generator=g)
        B = torch.randn(Nr, D, device=dev, generator=g)
        out = torch.zeros(2, dtype=torch.float64, device=dev)
        nb = lib.sumac_relu_bat_reduce_workspace_bytes(M, Nr, D, prec)
        if nb == 0:
            continue
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)

        def launch():
            _native.check(lib.sumac_relu_bat_reduce(P(A), P(B), M, Nr, D, P(out), prec, P(ws), nb,
                                                    P(err), stream), "relu_bat_reduce")
        for _ in range(3):
            launch()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(20):
            launch()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 20
        tf = (M * Nr * (2 * D - 1) + 3 * M * Nr) / (ms * 1e-3) / 1e12
        res[f"D{D}"] = {"ms": ms, "tflops": tf, "frac_tf32": tf / tf32_peak}
    _native.raise_device_error(dev)
    return res


def _teardown(st, world):
    """Free the CUDA graph (it holds captured NCCL collectives) before the communicator goes,
    then leave together: every rank reaches the barrier, then destroys the process group."""
    st.graph = None
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------ CPU arms
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def import_reference():
    """The unmodified reference package installed in baseline/_ref (pip --target), imported with
    TorchDynamo disabled (its torch.compile wrappers then run eagerly on the CPU)."""
    os.environ["TORCHDYNAMO_DISABLE"] = "1"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import sumac  # noqa: F401
    if not os.path.abspath(sumac.__file__).startswith(REF_DIR):
        raise ImportError(f"sumac resolved to {sumac.__file__}, not baseline/_ref")
    return sumac


class ReferenceSalsaSample:
    """The reference's own CPU SALSA path on the workload (training/salsa.py:212-316 with
    config.device = cpu): pruning, init_salsa_factors, the two StochasticRowBlockDatasets, and
    update_factor_salsa with the kernel get_tunable_kernel(cfg) selects on the CPU (the torch
    fallback relu(B A^T) C). A step is one block-update pair (B, then A), 1/num_blocks of an
    iteration; the per-iteration reshuffle of both datasets is timed once and added pro rata."""

    def __init__(self, idx_np, val_np, shape, d, nb):
        import_reference()
        from sumac import AutotuneMode, SumacConfig, SumacMethod
        from sumac.data import prune_zero_rows_cols
        from sumac.datasets import StochasticRowBlockDataset
        from sumac.kernels.tuning import get_tunable_kernel
        from sumac.training.salsa import init_salsa_factors, update_factor_salsa
        torch.set_num_threads(os.cpu_count())
        self.update = update_factor_salsa
        S_index = torch.from_numpy(idx_np)
        self.S_value = torch.from_numpy(val_np)
        S_index, _, _, m, n = prune_zero_rows_cols(S_index, shape)
        self.cfg = SumacConfig(method=SumacMethod.SALSA, rank=d, num_blocks=nb, seed=0,
                               verbose=False, autotune=AutotuneMode.DISABLE,
                               device=torch.device("cpu"))
        gen, gen_rows, gen_cols = self.cfg.get_generator()
        self.A, self.B = init_salsa_factors(S_index, self.S_value, m, n, d, gen=gen)
        self.dA, self.dB = torch.zeros_like(self.A), torch.zeros_like(self.B)
        self.S_index, self.S_index_T = S_index, S_index[[1, 0], :]
        self.ds_rows = StochasticRowBlockDataset(S_index, self.S_value, m, nb, gen=gen_rows)
        self.ds_cols = StochasticRowBlockDataset(self.S_index_T, self.S_value, n, nb, gen=gen_cols)
        self.kernel = get_tunable_kernel(self.cfg)
        self.momentum = torch.tensor(self.cfg.momentum, dtype=self.A.dtype)
        self.lrate = torch.tensor(self.cfg.learning_rate, dtype=self.A.dtype)
        self.nb = nb
        self.step_no = 0
        t0 = time.perf_counter()
        self.ds_rows.reshuffle()
        self.ds_cols.reshuffle()
        self.reshuffle_s = time.perf_counter() - t0

    def pair_seconds(self):
        k = self.step_no % self.nb
        self.step_no += 1
        unbias = 1 - self.momentum ** self.step_no
        t0 = time.perf_counter()
        self.B, self.dB = self.update(self.kernel, self.S_index, self.S_value, self.ds_rows, k,
                                      self.A, self.B, self.dB, self.momentum, unbias, self.lrate)
        self.A, self.dA = self.update(self.kernel, self.S_index_T, self.S_value, self.ds_cols, k,
                                      self.B, self.A, self.dA, self.momentum, unbias, self.lrate)
        return time.perf_counter() - t0

    def iter_per_s(self, pair_times):
        mean = sum(pair_times) / len(pair_times)
        return 1.0 / (self.nb * mean + self.reshuffle_s), mean


def cpu_baseline(args, idx_np, val_np, shape, d, nb):
    """The reference's own CPU path on a bounded sample: 3 block-update pairs after 1 untimed."""
    try:
        ref = ReferenceSalsaSample(idx_np, val_np, shape, d, nb)
    except ImportError as e:
        return {"value": None, "unit": "iter/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": f"not run: the reference could not be imported ({e})"}
    ref.pair_seconds()
    times = [ref.pair_seconds() for _ in range(3)]
    value, mean = ref.iter_per_s(times)
    return {"value": value, "unit": "iter/s", "cores": torch.get_num_threads(), "kind": "reference",
            "cpu_model": cpu_model(),
            "sample": f"3 SALSA block-update pairs ({mean:.2f} s each, 1/{nb} of an iteration) of the "
                      f"reference's update_factor_salsa on the CPU (torch fallback kernels, fp32) "
                      f"plus one reshuffle of both datasets ({ref.reshuffle_s:.2f} s), scaled to "
                      f"iterations/s"}


def bench_config(cfgd, m, n, nnz, world, args):
    """The `config` object of the JSON line, identical in both arms."""
    return {"workload": cfgd["desc"], "m_eff": m, "n_eff": n, "nnz": int(nnz),
            "rank": cfgd["rank"], "num_blocks": cfgd["num_blocks"],
            "method": cfgd.get("method", "SALSA"),
            "parallelism": "single GPU" if world == 1 else
            f"rows of A and B sharded over {world} GPUs (NCCL allreduce of each block's fixed rows)",
            "l2": "inputs larger than L2 (CSR of both directions ~0.3 GB per step)"}


def run_reference(args):
    rank, world, local = dist_info()
    if rank != 0:
        return
    cfgd = CONFIGS[args.config]
    if cfgd.get("method") == "GD":
        print(json.dumps({"impl": "reference", "unavailable": "C5 does not fit the host's dense "
                          "fallbacks (a 32 GB block product in fp32)"}))
        return
    idx_np, val_np, shape = MAKERS[args.config]()
    d, nb = cfgd["rank"], cfgd["num_blocks"]
    try:
        ref = ReferenceSalsaSample(idx_np, val_np, shape, d, nb)
    except ImportError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"the reference in baseline/_ref "
                          f"could not be imported: {e}"}))
        return
    m, n = ref.A.shape[0], ref.B.shape[0]
    for _ in range(args.warmup):
        ref.pair_seconds()
    times = [ref.pair_seconds() for _ in range(args.steps)]
    value, mean = ref.iter_per_s(times)
    print(json.dumps({
        "impl": "reference", "metric": "fused ReLU(AB^T)-reduce TFLOP/s; GD/SALSA iters/s at 1/2/4/8 B200",
        "value": value, "unit": "iter/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded stand-in)",
        "config": bench_config(cfgd, m, n, val_np.size, world, args),
        "cpu_baseline": {"value": value, "unit": "iter/s", "cores": torch.get_num_threads(),
                         "cpu_model": cpu_model(), "kind": "reference",
                         "sample": f"each step = one SALSA block-update pair ({mean:.2f} s mean) of "
                                   f"the reference's own update_factor_salsa on the CPU "
                                   f"(sumac_factorize's CPU path, torch fallback kernels), "
                                   f"1/{nb} of an iteration; plus one reshuffle of both datasets "
                                   f"({ref.reshuffle_s:.2f} s) per iteration"},
        "e2e": {"value": value, "unit": "iter/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_gd(args):
    """GD epochs per second on one GPU with the data resident (C5): each step is one pass over
    the 123 row blocks (block gradients through the fused product passes, one Adam step per
    block). Algorithmic work 6 m n d per epoch (L, grad A, grad B)."""
    from sumac_b200 import SumacConfig, SumacMethod, _native
    from sumac_b200.data import prune_zero_rows_cols
    from sumac_b200.gd import GDState
    from sumac_b200.salsa import init_salsa_factors
    rank, world, local = dist_info()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    cfgd = CONFIGS[args.config]
    idx_np, val_np, shape = MAKERS[args.config]()
    d, nb = cfgd["rank"], cfgd["num_blocks"]
    S_index = torch.from_numpy(idx_np).to(dev)
    S_value = torch.from_numpy(val_np).to(dev)
    del idx_np
    S_index, _, _, m, n = prune_zero_rows_cols(S_index, shape)
    cfg = SumacConfig(method=SumacMethod.GD, rank=d, num_blocks=nb, seed=0, verbose=False,
                      allow_tf32=args.precision == "tf32", device=dev)
    gen, gen_blocks, gen_loader = cfg.get_generator()
    A, B = init_salsa_factors(S_index, S_value, m, n, d, gen)
    if world > 1:
        from sumac_b200.shard import ShardedGDState
        st = ShardedGDState(S_index, S_value, m, n, cfg, A, B, gen_blocks, gen_loader)
    else:
        st = GDState(S_index, S_value, m, n, cfg, A, B, gen_blocks, gen_loader)
    del A, B
    for _ in range(args.warmup):
        st.epoch(False)
    torch.cuda.synchronize()
    _native.raise_device_error(dev)
    if world > 1:
        dist.barrier()
    lib = _native.lib()
    launches0 = lib.sumac_kernel_launches()
    ev0, ev1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            st.epoch(False)
        ev1.record()
        torch.cuda.synchronize()
    _native.raise_device_error(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    launches = lib.sumac_kernel_launches() - launches0
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    flops = 6.0 * m * n * d
    tf = flops / (ms * 1e-3) / 1e12
    pk = peaks()
    tf32_peak = pk["bf16_tflops"] / 2.0
    print(json.dumps({
        "metric": "GD epochs/s (C5)", "value": 1e3 / ms, "unit": "epoch/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "tf32" if args.precision == "tf32" else "f32 (3xTF32)",
        "data": "synthetic (seeded stand-in)",
        "config": {"workload": cfgd["desc"], "m_eff": m, "n_eff": n, "nnz": int(val_np.size),
                   "rank": d, "num_blocks": nb, "method": "GD",
                   "parallelism": "single GPU" if world == 1 else
                   f"each step's row block split over {world} GPUs (NCCL allreduce of grad B)",
                   "l2": "inputs larger than L2 (factors 256 MB each, CSR 3.2 GB)"},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": tf32_peak, "unit": "TFLOP/s",
                     "frac": tf / tf32_peak, "traffic": None,
                     "note": "achieved = 6 m n d per epoch (algorithmic); the fused passes "
                             "recompute L, doing 8 m n d"},
        "cpu_baseline": None, "cpu_note": "not run on CPU: C5 does not fit the host's dense "
                                          "fallbacks (a 32 GB block product in fp32)",
        "e2e": None, "clocks": clk.summary(),
        "gpu_launches": int(launches),
    }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_product_only(args):
    """The fused product alone at one block update's shapes (rows of the updated factor x one block
    of the fixed factor), random operands: a small, self-contained case for profiling."""
    from sumac_b200 import _native, ops
    dev = torch.device("cuda", 0)
    cfgd = CONFIGS[args.config]
    d, nb = cfgd["rank"], cfgd["num_blocks"]
    M = {"c4": 138963, "c3": 50000, "c2": 70000}[args.config]
    b = (M + nb - 1) // nb
    prec = 1 if args.precision == "tf32" else 3
    Dp = ops.padded_rank(d)
    g = torch.Generator(device=dev).manual_seed(0)
    X = torch.zeros((M, Dp), device=dev)
    X[:, :d] = torch.randn(M, d, device=dev, generator=g)
    F = torch.zeros((b, Dp), device=dev)
    F[:, :d] = torch.randn(b, d, device=dev, generator=g)
    ldct = (b + 3) // 4 * 4
    Ct = torch.zeros((Dp, ldct), device=dev)
    Ct[:d, :b] = torch.randn(d, b, device=dev, generator=g)
    hi = lambda t: (t.view(torch.int32) & -8192).view(torch.float32)  # noqa: E731
    Fhi, Flo = (hi(F), F - hi(F)) if prec == 3 else (tf32_round(F), None)
    Chi, Clo = (hi(Ct), Ct - hi(Ct)) if prec == 3 else (Ct, None)
    lib = _native.lib()
    splits = lib.sumac_relu_product_splits(M, b, Dp, prec)
    part = torch.empty(splits * M * Dp + 16, device=dev)
    P = _native.ptr
    err = _native.err_word(dev)

    def launch():
        _native.check(lib.sumac_relu_product(P(X), M, P(Fhi), P(Flo), P(Chi), P(Clo), ldct, b,
                                             Dp, prec, P(part), P(err),
                                             _native.stream_ptr(dev)), "relu_product")
    for _ in range(args.warmup):
        launch()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(args.steps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    _native.raise_device_error(dev)
    ms = e0.elapsed_time(e1) / args.steps
    tflops = 4.0 * M * b * d / (ms * 1e-3) / 1e12
    ref = torch.relu(X[:, :d] @ F[:, :d].T) @ Ct[:d, :b].T
    err_rel = float((part[:splits * M * Dp].view(splits, M, Dp).sum(0)[:, :d] - ref).abs().max() / ref.abs().max())
    print(json.dumps({"product_only": args.config, "M": M, "N": b, "d": d, "precision": prec,
                      "ms_per_launch": ms, "tflops": tflops, "max_rel_err_vs_torch": err_rel}))


def run_profile_iteration(args):
    """One eager SALSA iteration at the workload's shapes (both CSR rebuilds and 2 x num_blocks
    block updates as separate launches, no CUDA graph), after the setup: a short, self-contained
    command for kernel profiles of the iteration's kernels."""
    from sumac_b200 import SumacConfig, SumacMethod, _native
    from sumac_b200.data import prune_zero_rows_cols
    from sumac_b200.salsa import SalsaState, draw_perm, init_salsa_factors
    dev = torch.device("cuda", 0)
    cfgd = CONFIGS[args.config]
    idx_np, val_np, shape = MAKERS[args.config]()
    S_index = torch.from_numpy(idx_np).to(dev)
    S_value = torch.from_numpy(val_np).to(dev)
    S_index, _, _, m, n = prune_zero_rows_cols(S_index, shape)
    cfg = SumacConfig(method=SumacMethod.SALSA, rank=cfgd["rank"], num_blocks=cfgd["num_blocks"],
                      seed=0, verbose=False, allow_tf32=args.precision == "tf32", device=dev)
    gen, gen_rows, gen_cols = cfg.get_generator()
    A, B = init_salsa_factors(S_index, S_value, m, n, cfg.rank, gen)
    st = SalsaState(S_index, S_value, m, n, cfg, A, B)
    st.use_graph = False
    st.iteration(1, draw_perm(m, gen_rows, dev), draw_perm(n, gen_cols, dev))
    torch.cuda.synchronize()
    _native.raise_device_error(dev)
    print(json.dumps({"profile_iteration": args.config, "m": m, "n": n}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c4")
    ap.add_argument("--precision", choices=["tf32", "3xtf32"], default="tf32")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--product-only", action="store_true",
                    help="time the fused product alone at one block update's shapes")
    ap.add_argument("--profile-iteration", action="store_true",
                    help="run one eager SALSA iteration (for kernel profiles) and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_iteration:
        run_profile_iteration(args)
    elif args.product_only:
        run_product_only(args)
    elif args.impl == "ours" and CONFIGS[args.config].get("method") == "GD":
        run_gd(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
