"""Benchmark of the bfp16 weight-GEMM hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU, NCCL)
    python bench.py --case <name> [--iters I]              (one kernel or DiT block on its config shape: ncu target)

Workload (config 1, the DiT FFN up-projection): X[4352, 3072] ~ N(0,1) bf16, W[3072, 12288] ~ N(0, 0.02) packed to
bfp16, bias ~ N(0, 0.01); one step = quantise X to bfp16 (bit-exact with the reference) + the packed-weight GEMM with
the bias epilogue, fp32 accumulation, bf16 out. The metric is the reference's headline "bfp16 GEMM TFLOP/s"
(2*M*N*K per step, quantiser time included). On N GPUs the one GEMM is split by weight columns (strong scaling):
GPU g streams the contiguous bytes of its N/N_gpu columns of the packed W (no repacking) and writes C[:, its
columns]; every GPU quantises the whole X itself, and no collective runs in the step. Inputs rotate over enough
independent sets that the bytes touched between two uses of a set exceed the 126 MB L2.

--impl reference times the reference's own CPU path (its numpy bfp16 quantisation + decode + float32 matmul,
restated in oracle/bfp16_oracle.py) on all host cores: the full config-1 rows per step when the run fits a few
minutes, else a row sample.
"""

import argparse
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def _wants_reference(argv):
    return any(a == "--impl=reference" for a in argv) or any(
        a == "--impl" and i + 1 < len(argv) and argv[i + 1] == "reference" for i, a in enumerate(argv))


if _wants_reference(sys.argv):
    # the reference's numpy path on every host core the process may use, whatever a launcher (torchrun sets
    # OMP_NUM_THREADS=1) put in the environment; BLAS reads these when numpy is first imported
    _cores = str(len(os.sched_getaffinity(0)))
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = _cores

M, K, N = 4352, 3072, 12288
FLOP = 2.0 * M * N * K
WORKLOAD = "C1: bfp16 linear X[4352,3072] @ W[3072,12288] + bias, bf16 out (DiT FFN up-projection)"
METRIC = "bfp16 GEMM TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126e6
BF16_OUT_TOL = 2e-3 + 2.0 ** -8       # the GEMM parity bar of the tests: the north-star 2e-3 + the bf16 output step
COS_BAR = 0.999


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="reference arm: X rows per step (0 = all 4352 when the run fits ~3 minutes, else a sample)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 2-5 measurements")
    ap.add_argument("--case", default=None, help="run one profiling case and exit (see CASES)")
    ap.add_argument("--iters", type=int, default=3)
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def ncu_traffic():
    """dram read+write bytes per launch of the config-1 GEMM, from the committed ncu summary (None if absent)."""
    p = os.path.join(ROOT, "profiles", "bfp16_linear_c1.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every ~5 ms while the timed region runs."""

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h) if hasattr(
                    nv, "nvmlDeviceGetCurrentClocksEventReasons") else nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for bit, name in ((0x8, "hw_slowdown"), (0x40, "hw_thermal_slowdown"), (0x20, "sw_thermal_slowdown"),
                                  (0x4, "sw_power_cap"), (0x80, "hw_power_brake_slowdown")):
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.nv:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2], "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(s)}


def dist_init():
    os.environ.pop("NCCL_DEBUG", None)   # rank 0's stdout carries exactly one JSON line (no NCCL banner)
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


# ------------------------------------------------------------------------------------------------------------------
# the reference's CPU path (oracle/bfp16_oracle.py restates it): cpu_baseline of our line and the --impl reference arm
# ------------------------------------------------------------------------------------------------------------------

def _blas_threads():
    """Pin the BLAS pool to every host core the process may use (threadpoolctl, if importable) and return the count."""
    cores = len(os.sched_getaffinity(0))
    try:
        import threadpoolctl
        threadpoolctl.threadpool_limits(limits=cores, user_api="blas")
    except Exception:
        pass
    return cores


class ReferenceCPU:
    """Config 1 on the host: W packed and decoded once (the resident weights), then per step
    to_bfp16(a_layout(X)) -> from_bfp16 -> a_unlayout -> float32 matmul with the bias."""

    def __init__(self, xsets=3, rows=M):
        import numpy as np
        from oracle import bfp16_oracle as O
        self.O, self.np = O, np
        self.cores = _blas_threads()
        rng = np.random.default_rng(0)
        W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        self.wd = O.unpack_b(O.pack_b(W), K, N)
        self.bias = O.bf16_round((rng.standard_normal(N) * 0.01).astype(np.float32))
        self.xs = [O.bf16_round(rng.standard_normal((M, K)).astype(np.float32)) for _ in range(xsets)]

    def step(self, i, rows):
        O = self.O
        x = self.xs[i % len(self.xs)][:rows]
        if rows % 128 == 0:
            xd = O.a_unlayout(O.from_bfp16(O.to_bfp16(O.a_layout(x, 128, 64))).astype(self.np.float32), rows, K)
        else:
            xd = O.quantize_rows(x)[1]
        return O.linear(xd, self.wd, self.bias)


def cpu_baseline_sample():
    """The reference's CPU path on config 1 in full, once (after one 128-row warm-up): (TFLOP/s, seconds, threads)."""
    ref = ReferenceCPU(xsets=1)
    ref.step(0, 128)
    t = time.perf_counter()
    ref.step(0, M)
    dt = time.perf_counter() - t
    return FLOP / dt / 1e12, dt, ref.cores


def cpu_dit_block_sample():
    """The DiT step's host path (the CPU oracle of the block math, oracle/dit_oracle.py, numpy on every host core) on
    config 4's shapes with one block, once: seconds (the embedding, one block and the projection; a 32-block step
    is estimated as 32 x this), and the thread count."""
    import numpy as np
    import torch
    from oracle import dit_oracle as DO
    from redline_tiny_b200 import dit, host_glue as HG
    cfg = dit.DiTConfig(blocks=1)
    prep = DO.prepare(dit.random_weights(cfg, seed=0, device="cpu"))
    rng = np.random.default_rng(0)
    lat = rng.standard_normal((cfg.image, cfg.latent_ch)).astype(np.float32)
    txt = rng.standard_normal((cfg.text, cfg.hidden)).astype(np.float32)
    t = time.perf_counter()
    DO.forward(cfg, prep, lat, txt, HG.SIGMAS[3], HG)
    return time.perf_counter() - t, _blas_threads()


def run_reference(args, ws, rank):
    if rank != 0:          # under torchrun rank 0 alone times the host path; the others exit without work
        return
    ref = ReferenceCPU()
    rows = args.ref_rows
    if rows <= 0:
        ref.step(0, 128)
        t = time.perf_counter()
        ref.step(1, 128)
        full = (time.perf_counter() - t) * M / 128
        budget = 150.0
        if (args.steps + args.warmup) * full <= budget:
            rows = M
        else:
            rows = max(128, min(M, int(budget / (args.steps + args.warmup) / full * M) // 128 * 128))
    for i in range(args.warmup):
        ref.step(i, rows)
    t = time.perf_counter()
    for i in range(args.steps):
        ref.step(i, rows)
    dt = time.perf_counter() - t
    value = 2.0 * rows * N * K * args.steps / dt / 1e12
    out = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": ws,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
           "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic",
           "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N, "parallelism": "host cores (rank 0 only)",
                      "rows_per_step": rows, "same_config": rows == M},
           "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": ref.cores, "kind": "port",
                            "sample": f"{rows} of {M} rows of X per step (to_bfp16(a_layout) + from_bfp16 + float32 "
                                      f"matmul with bias vs the decoded packed W, numpy/OpenBLAS on {ref.cores} "
                                      f"threads)"},
           "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------------------------------------------------------
# helpers on the GPU
# ------------------------------------------------------------------------------------------------------------------

def _event_ms(fn, n, w, stream):
    import torch
    for _ in range(w):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def _max_over_ranks(vals, dev, ws):
    """Element-wise max of a list of floats over the ranks (the list itself on one GPU)."""
    if ws == 1:
        return list(vals)
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm()))


def _max_rel(got, ref):
    return float((got.double() - ref.double()).abs().max() / ref.double().abs().max())


def decoded_weight(W):
    """Float B (K, N) on the GPU -> its bfp16-decoded values (K, N) float32: the quantiser on B^T's rows (blocks of 8
    consecutive K of one column, the blocks pack_b forms)."""
    from redline_tiny_b200 import ops
    _, dq = ops.quantize_bfp16(W.t().contiguous(), want_bytes=False)
    return dq.t().float()


def gemm_parity(dq, W, bias, w_full, w_shard, n0, gemm, stream, ws):
    """The step's GEMM (gemm(): this GPU's columns, through the split-K workspace when the shape splits) on one input
    set against (a) the same columns computed unsplit (a split changes only the order of fp32 additions: max-rel
    <= 2^-8, the bf16 step), (b) unsplit, the unsharded GEMM's columns [n0, n0 + n), bit for bit (N > 1), and (c) a
    float32 product of the decoded operands on 64 sampled rows (torch; TF32 off), max-rel <= the tests' bar.
    Returns (b, (a), (c))."""
    import torch
    from redline_tiny_b200 import _lib as L
    n = w_shard.N
    out = gemm()

    def whole(w, cols, b):
        c = torch.empty((M, cols), dtype=torch.bfloat16, device=dq.device)
        L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), cols, b.data_ptr(), L.RL_EPI_BIAS,
               c.data_ptr(), L.RL_BF16, stream.cuda_stream)
        return c
    mine = whole(w_shard, n, bias[n0:n0 + n].contiguous())
    sched = _max_rel(out.float(), mine.float())
    equal = None
    if ws > 1:
        equal = bool(torch.equal(mine, whole(w_full, N, bias)[:, n0:n0 + n]))
    rows = torch.linspace(0, M - 1, 64, device=dq.device).round().long()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = dq[rows].float() @ decoded_weight(W)[:, n0:n0 + n] + bias[n0:n0 + n].float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return equal, sched, _max_rel(out[rows].float(), ref)


def launch_breakdown(model, fn, stream):
    """Per-launch device time of one call of fn (a DiT step): a CUDA event after every C-ABI call and every NCCL
    collective (the events themselves add a few percent to the step). Returns ({entry point: [launches, ms]},
    [(launch, us) of block 10])."""
    import torch
    import torch.distributed as dist
    from redline_tiny_b200 import _lib as L
    marks = []

    def mark(name):
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        marks.append((name, e))

    call = L.call
    colls = {n: getattr(dist, n) for n in ("all_reduce", "reduce_scatter_tensor", "all_gather_into_tensor")}

    def timed_call(name, *a):
        r = call(name, *a)
        mark(name[3:] if name.startswith("rl_") else name)
        return r

    def timed(n):
        def f(*a, **k):
            r = colls[n](*a, **k)
            mark("nccl_" + n)
            return r
        return f
    L.call = timed_call
    for n in colls:
        setattr(dist, n, timed(n))
    try:
        mark("start")
        fn()
        torch.cuda.synchronize()
    finally:
        L.call = call
        for n, f in colls.items():
            setattr(dist, n, f)
    seq = [(n1, e0.elapsed_time(e1) * 1e3) for (_, e0), (n1, e1) in zip(marks, marks[1:])]
    totals = {}
    for name, us in seq:
        t = totals.setdefault(name, [0, 0.0])
        t[0] += 1
        t[1] += us / 1e3
    # a block starts at its QKV projection: qkv_linear (fused), or the linear before qkv_post
    starts = [i - (2 if seq[i - 1][0] == "qkv_post" else 1) for i, (name, _) in enumerate(seq) if name == "attention"]
    block = seq[starts[10]:starts[11]] if len(starts) > 11 else []
    return {k: [v[0], round(v[1], 3)] for k, v in totals.items()}, [(k, round(v, 1)) for k, v in block]


# ------------------------------------------------------------------------------------------------------------------
# configs 2-5 and the paths beyond them
# ------------------------------------------------------------------------------------------------------------------

def measure_next_rows(dev, stream, seed):
    """The paths beyond configs 1-5 (CUDA events, seeded synthetic inputs, random N(0, 0.02) weights): the VAE
    decoder's 3x3 convolutions at two of its stages (vae_decode.py:311-348: 1152 channels at 128^2, 288 at 512^2 -
    K = 9 taps x 288 channels, each padded to 320) and one Qwen3-VL-8B decoder layer at the reference's M = 1536 rows
    (vlm_run.py:396-431, causal GQA over 1500 valid rows)."""
    import math
    import torch
    from redline_tiny_b200 import ops, vlm
    from redline_tiny_b200 import _lib as L
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 5)
    res = {}
    for H, C in ((128, 1152), (512, 288)):
        x = ops.quantize_bfp16(torch.randn((H * H, C), generator=g, device=dev), want_bytes=False)[1].view(H, H, C)
        w = torch.randn((C, C, 3, 3), generator=g, device=dev) * 0.02
        pw, bias, taps = ops.conv_weight(w, torch.randn(C, generator=g, device=dev) * 0.01)
        y = torch.empty((H, H, pw.N), dtype=torch.bfloat16, device=dev)
        ms = _event_ms(lambda: ops.conv2d(x, pw, bias, taps, out=y), 10, 3, stream)
        fl = 2.0 * H * H * 9 * C * C
        res[f"vae_conv3_{H}x{H}x{C}"] = {"ms": ms, "TFLOP/s": fl / (ms * 1e-3) / 1e12, "GFLOP": fl / 1e9,
                                         "gather_bytes": L.lib().rl_conv2d_workspace(H, H, C, 3),
                                         "path": "implicit GEMM (3-D TMA from the image)"
                                         if L.lib().rl_conv2d_workspace(H, H, C, 3) == 0 else "im2col + GEMM"}
        del x, w, pw, y
    cfg = vlm.LMConfig()
    Mv, valid = 1536, 1500
    lm = vlm.LM(cfg, vlm.random_lm_weights(cfg, seed=seed), Mv, device=dev)
    ang = torch.rand((Mv, 64), generator=g, device=dev) * 2 * math.pi
    lm.set_positions(torch.cos(ang).cpu(), torch.sin(ang).cpu(), valid)
    lm.load_x(torch.randn((Mv, cfg.hidden), generator=g, device=dev))
    ms = _event_ms(lambda: lm.layer(0), 10, 3, stream)
    fl = cfg.flop_per_layer(Mv, valid)
    res["vlm_layer_m1536"] = {"ms": ms, "TFLOP/s": fl / (ms * 1e-3) / 1e12, "GFLOP": fl / 1e9}
    del lm
    torch.cuda.empty_cache()
    L.device_status()      # raises if any kernel recorded a device-side error (e.g. a bounded wait that ran out)
    return res


def measure_gemm_sweep(dev, stream, ws, rank, g):
    """Config 5's GEMM sweep, K = 3072, N = 12288, M in {256, 1024, 4352, 17408}: one GEMM split by weight columns
    over the N GPUs (strong scaling; each GPU its N / N_gpu contiguous columns); ms = the slowest GPU's."""
    import torch
    from redline_tiny_b200 import ops
    from redline_tiny_b200 import _lib as L
    K5, N5 = 3072, 12288
    ws5 = [ops.PackedWeight.from_float(torch.randn((K5, N5), generator=g, device=dev) * 0.02) for _ in range(2)]
    shards = [w.shard(rank, ws)[0] for w in ws5]
    n0 = ws5[0].shard(rank, ws)[1]
    nloc = N5 // ws
    bias = (torch.randn((N5,), generator=g, device=dev) * 0.01).to(torch.bfloat16)[n0:n0 + nloc].contiguous()
    res, split = {}, {}
    for Ms in (256, 1024, 4352, 17408):
        xs = [ops.quantize_bfp16(torch.randn((Ms, K5), generator=g, device=dev).to(torch.bfloat16),
                                 want_bytes=False)[1] for _ in range(2)]
        c = torch.empty((Ms, nloc), dtype=torch.bfloat16, device=dev)
        gws = ops.gemm_workspace(Ms, K5, nloc, dev, epilogue=L.RL_EPI_BIAS)
        wptr, wbytes = (0, 0) if gws is None else (gws.data_ptr(), gws.numel())
        it = [0]

        def f():
            i = it[0] = it[0] + 1
            L.call("rl_linear_bfp16_ws", xs[i % 2].data_ptr(), Ms, K5, shards[i % 2].native.data_ptr(), nloc,
                   bias.data_ptr(), L.RL_EPI_BIAS, c.data_ptr(), L.RL_BF16, wptr, wbytes, stream.cuda_stream)
        res[str(Ms)] = _event_ms(f, 20, 3, stream)
        split[str(Ms)] = gws is not None
        del xs, c, gws
    mx = _max_over_ranks([res[k] for k in res], dev, ws)
    out = {}
    for (k, _), ms in zip(list(res.items()), mx):
        Ms = int(k)
        out[k] = {"ms": ms, "TFLOP/s": 2.0 * Ms * N5 * K5 / (ms * 1e-3) / 1e12, "split_k": split[k]}
    out["split"] = f"N/{ws} = {nloc} weight columns per GPU (strong scaling; ms of the slowest GPU)"
    return out


def measure_configs(dev, stream, ws, rank):
    """The other benchmark configs (2-5) and the parity checks of the partitioned DiT paths. CUDA-event timed; inputs
    are seeded synthetic tensors of the configs' shapes; weights N(0, 0.02)."""
    import torch
    from redline_tiny_b200 import dit, ops
    from redline_tiny_b200 import host_glue as HG
    from redline_tiny_b200 import _lib as L
    g = torch.Generator(device=dev)
    g.manual_seed(100 + rank)
    out, failures = {}, []
    out["C5_gemm_sweep_K3072_N12288"] = measure_gemm_sweep(dev, stream, ws, rank, g)
    # the quantiser alone at config 1's X (HBM-bound): bf16 in, bfp16 bytes (row-major blocks) and the decoded bf16
    # copy the GEMM reads out; inputs rotate over 3 sets of 26.7 MB, outputs over 2 (together above the 126 MB L2)
    Mq, Kq = 4352, 3072
    xs = [torch.randn((Mq, Kq), generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
    qs = [torch.empty(Mq * Kq // 8 * 9, dtype=torch.uint8, device=dev) for _ in range(2)]
    ds = [torch.empty((Mq, Kq), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    iq = [0]

    def fq():
        i = iq[0] = iq[0] + 1
        L.call("rl_quantize_bfp16", xs[i % 3].data_ptr(), L.RL_BF16, Mq, Kq, L.RL_ROWMAJOR, qs[i % 2].data_ptr(),
               ds[i % 2].data_ptr(), stream.cuda_stream)
    ms = _event_ms(fq, 50, 5, stream)
    nbytes = Mq * Kq * (2 + 9 / 8 + 2)
    pk, kind = peaks()
    out["quantize_c1"] = {"ms": ms, "GB/s": nbytes / (ms * 1e-3) / 1e9, "bytes": nbytes,
                          "frac_of_hbm": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], "peak_kind": kind}
    del xs, qs, ds
    # config 2: Qwen3-VL SwiGLU MLP, X[512, 4096] -> gate/up [4096, 12288] -> down [12288, 4096]
    M2, K2, F2, N2 = 512, 4096, 12288, 4096
    wu = ops.PackedWeight.from_float(torch.randn((K2, 2 * F2), generator=g, device=dev) * 0.02, swiglu=True)
    wd = ops.PackedWeight.from_float(torch.randn((F2, N2), generator=g, device=dev) * 0.02)
    x2 = torch.randn((M2, K2), generator=g, device=dev).to(torch.bfloat16)
    o2 = torch.empty((M2, N2), dtype=torch.bfloat16, device=dev)
    wsp = torch.empty(L.lib().rl_swiglu_mlp_workspace(M2, K2, F2, 0), dtype=torch.uint8, device=dev)
    ms = _event_ms(lambda: ops.swiglu_mlp(x2, wu, wd, out=o2, workspace=wsp), 20, 3, stream)
    fl = 2.0 * M2 * K2 * 2 * F2 + 2.0 * M2 * F2 * N2
    out["C2_swiglu_mlp"] = {"ms": ms, "TFLOP/s": fl / (ms * 1e-3) / 1e12, "weights_MB": 169.87,
                            "down_gemm_split_k": L.lib().rl_linear_bfp16_workspace(M2, F2, N2, 0) > 0}
    del wu, wd, wsp
    # configs 3 and 4: the DiT (hidden 3072, 24 x 128 heads, FFN 12288, 256 text + 4096 image tokens); the weights
    # are the same on every rank (seed 1000), so the tensor-parallel step below can be checked against this model
    cfg = dit.DiTConfig()
    model = dit.DiT(cfg, dit.random_weights(cfg, seed=1000))
    lat = torch.randn((cfg.image, cfg.latent_ch), generator=g, device=dev)
    txt = torch.randn((cfg.text, cfg.hidden), generator=g, device=dev)
    model.set_t(0.5)
    model.embed(lat, txt)
    b0 = model.blocks[0]

    def sublayer():   # config 3: the joint-attention sublayer (QK-RMSNorm + RoPE in the QKV GEMM's epilogue)
        L.call("rl_qkv_linear", model.a.data_ptr(), cfg.M, cfg.hidden, b0["qkv"].native.data_ptr(), cfg.heads,
               cfg.heads, model.rope_cs.data_ptr(), b0["wq"].data_ptr(), b0["wk"].data_ptr(), model.q.data_ptr(),
               model.k.data_ptr(), model.vt.data_ptr(), model.ldv, stream.cuda_stream)
        L.call("rl_attention", model.q.data_ptr(), model.k.data_ptr(), model.vt.data_ptr(), model.ldv, cfg.heads,
               cfg.M, cfg.M, cfg.M, None, 1.0, model.o.data_ptr(), cfg.hidden, stream.cuda_stream)
        model._linear(model.o, b0["o"], model.c)
    ms = _event_ms(sublayer, 10, 3, stream)
    Mt, D = cfg.M, cfg.hidden
    fl = 2.0 * Mt * D * 3 * D + 2.0 * Mt * D * D + 4.0 * cfg.heads * Mt * Mt * 128
    out["C3_joint_attention_sublayer"] = {"ms": ms, "TFLOP/s": fl / (ms * 1e-3) / 1e12, "GFLOP": fl / 1e9}

    ms = _event_ms(lambda: model.denoise_step(lat, txt, 3), 3, 2, stream)
    out["C4_dit_step"] = {"ms": ms, "TFLOP/s": cfg.flop_per_step() / (ms * 1e-3) / 1e12,
                          "TFLOP_per_step": cfg.flop_per_step() / 1e12, "weights_GB": 5.44}
    totals, block = launch_breakdown(model, lambda: model.denoise_step(lat, txt, 3), stream)
    out["C4_dit_step"]["launches_per_step"] = totals
    out["C4_dit_step"]["block10_us"] = block
    # the tensor-parallel check's reference velocity: this unsharded model on the TP inputs (seeds 7, 8)
    lat_tp = torch.randn((cfg.image, cfg.latent_ch), generator=torch.Generator(device=dev).manual_seed(7), device=dev)
    txt_tp = torch.randn((cfg.text, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(8), device=dev)
    v_ref = model.forward(lat_tp, txt_tp, HG.SIGMAS[3]).clone() if ws > 1 else None
    # the unsharded model's own sensitivity: its velocity when every text-state value moves by half a bf16 step
    # (+-2^-9 relative, random signs) - how far apart two roundings of the same computation can end up after 32
    # random-init blocks
    gp = torch.Generator(device=dev).manual_seed(9)
    sign = torch.randint(0, 2, txt_tp.shape, generator=gp, device=dev).float() * 2 - 1
    v_pert = model.forward(lat_tp, txt_tp * (1 + sign * 2.0 ** -9), HG.SIGMAS[3]).clone()   # forward returns a view
    floor = _cos(v_pert, model.forward(lat_tp, txt_tp, HG.SIGMAS[3]))
    out["C4_dit_step"]["velocity_cos_under_half_ulp_input_change"] = floor
    del v_pert, sign

    # config 5's data-parallel DiT: the 8-step denoise (forward.py:550-618: SIGMAS, Euler) of one 1024^2 image per
    # GPU, GPU r on seed r (latent N(0,1) [4096, 64], text states N(0,1) [256, 3072])
    def denoise8(seed):
        gl = torch.Generator(device=dev).manual_seed(2000 + seed)
        x = torch.randn((cfg.image, cfg.latent_ch), generator=gl, device=dev)
        t8 = torch.randn((cfg.text, cfg.hidden), generator=gl, device=dev)
        for i in range(len(HG.SIGMAS)):
            x = model.denoise_step(x, t8, i)
        return x
    denoise8(rank)
    torch.cuda.synchronize()
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    reps = 2
    for _ in range(reps):
        mine = denoise8(rank)
    e1.record(stream)
    torch.cuda.synchronize()
    ms8 = _max_over_ranks([e0.elapsed_time(e1) / reps], dev, ws)[0]
    if ws > 1:
        import torch.distributed as dist
        lats = [torch.empty_like(mine) for _ in range(ws)]
        dist.all_gather(lats, mine.contiguous())
    else:
        lats = [mine]
    same = []
    if rank == 0:          # the same seeds on one GPU (this one): every image must be bit-identical
        for r in range(ws):
            same.append(bool(torch.equal(lats[r], denoise8(r))))
        if not all(same):
            failures.append(f"DP DiT: images {[r for r, s in enumerate(same) if not s]} differ from a 1-GPU run")
    out[f"C5_dit_dp{ws}_8step"] = {
        "ms_per_image_8_steps": ms8, "images_per_s_all_gpus": ws * 1e3 / ms8, "steps": len(HG.SIGMAS),
        "batch": ws, "seeds": list(range(ws)),
        "bit_identical_to_1gpu": same if rank == 0 else None,
        "note": "one image per GPU, no collective in the step loop; ms of the slowest GPU"}
    del model
    torch.cuda.empty_cache()
    out["next_rows"] = measure_next_rows(dev, stream, 100 + rank)
    if ws > 1:   # config 4 again, tensor-parallel over all ranks at batch 1
        import torch.distributed as dist
        # the default reduction (the projection GEMM stores each row block of its partial into the memory of the
        # rank that owns those rows, the owner's LayerNorm adds them and stores its rows into every rank's next A
        # operand), and beside it the other forms: at 2 GPUs the peer all-reduce (the GEMM stores its whole partial
        # into the other rank, both LayerNorms add both) and NCCL's bf16 all-reduce, above 2 NCCL's bf16 all-reduce
        # and its reduce-scatter + all-gather; and NCCL's all-reduce of fp32 partials. Parity:
        # the TP velocity against the unsharded model's on the same weights and inputs. Partials rounded to bf16
        # before they are added move every branch value by up to half a bf16 step, and the unsharded model itself
        # moves as far when its text input moves by half a bf16 step (velocity_cos_under_half_ulp_input_change), so
        # those modes are held to twice that distance (1 - cos), capped at 0.999; fp32 partials leave only the order
        # of fp32 additions and are held to 0.999.
        v_modes = {}
        names = {"peer": "fused: GEMM peer stores + LayerNorm sum",
                 "peer_rs": "fused reduce-scatter (GEMM stores row blocks to their owners) + LayerNorm on M/N rows "
                            "+ all-gather (LayerNorm stores its rows to every rank)",
                 "rs": "NCCL reduce-scatter + LayerNorm on M/N rows + NCCL all-gather",
                 "bf16": "NCCL all-reduce, bf16 (LayerNorm replicated)",
                 "fp32": "NCCL all-reduce, fp32 partials (LayerNorm replicated)"}
        # "auto" is "peer_rs"; the other forms are timed and checked beside it
        for mode in (("auto", "peer", "bf16", "fp32") if ws == 2 else ("auto", "bf16", "rs", "fp32")):
            w = dit.random_weights(cfg, seed=1000)       # the same weights on every rank, then this rank's shard
            tp_model = dit.DiT(cfg, dit.shard_weights(w, cfg, rank, ws), device=dev, tp=(rank, ws, dist.group.WORLD),
                               reduce_dtype=mode)
            del w
            torch.cuda.empty_cache()
            dist.barrier()
            ms = _event_ms(lambda: tp_model.denoise_step(lat_tp, txt_tp, 3), 3, 2, stream)
            ms = _max_over_ranks([ms], dev, ws)[0]
            v = tp_model.forward(lat_tp, txt_tp, HG.SIGMAS[3]).clone()
            v_modes[mode] = v
            cos, err = _cos(v, v_ref), _max_rel(v, v_ref)
            dt = HG.SIGMAS[4] - HG.SIGMAS[3]     # the Euler step this velocity feeds (forward.py:58-61)
            lcos = _cos(lat_tp + dt * v, lat_tp + dt * v_ref)
            worst = _max_over_ranks([-cos, err, -lcos], dev, ws)
            key = f"C4_dit_step_tp{ws}" + {"auto": "", "peer": "_peer_allreduce", "peer_rs": "_peer_rs",
                                           "bf16": "_nccl_bf16", "rs": "_nccl_rs", "fp32": "_nccl_fp32"}[mode]
            bar = COS_BAR if mode == "fp32" else min(COS_BAR, 1.0 - 2.0 * (1.0 - floor))
            e = {"ms": ms, "TFLOP/s_all_gpus": cfg.flop_per_step() / (ms * 1e-3) / 1e12,
                 "reductions_per_step": 2 * cfg.blocks,
                 "partial_bytes": cfg.M * cfg.hidden * (4 if mode == "fp32" else 2),
                 "reduction": names[tp_model.reduce_dtype],
                 "velocity_cos_vs_1gpu": -worst[0], "velocity_max_rel_vs_1gpu": worst[1],
                 "latent_cos_vs_1gpu": -worst[2],
                 "parity_bar": f"latent after the Euler step: cosine >= {COS_BAR} (the north-star bar); velocity "
                               f"cosine >= {bar:.6f}, against the unsharded model on the same weights and inputs"}
            if -worst[0] < bar:
                failures.append(f"{key}: velocity cosine {-worst[0]:.6f} < {bar:.6f}")
            if -worst[2] < COS_BAR:
                failures.append(f"{key}: latent cosine {-worst[2]:.6f} < {COS_BAR}")
            if mode in ("auto", "peer"):
                totals, block = launch_breakdown(tp_model, lambda: tp_model.denoise_step(lat_tp, txt_tp, 3), stream)
                e["launches_per_step"] = totals
                e["block10_us"] = block
            out[key] = e
            tp_model.close()
            del tp_model
            torch.cuda.empty_cache()
        if ws == 2:
            same = bool(torch.equal(v_modes["peer"], v_modes["bf16"]))
            out[f"C4_dit_step_tp{ws}_peer_allreduce"]["peer_sum_equals_nccl_bf16_allreduce"] = same
            if not same:
                failures.append("TP-2: the peer reduction's velocity differs from NCCL's bf16 all-reduce")
    L.device_status()      # raises if any kernel recorded a device-side error
    return out, failures


# ------------------------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------------------------

def run_ours(args, ws, rank, local):
    import torch
    from redline_tiny_b200 import ops
    from redline_tiny_b200 import _lib as L

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    n0, ncols, _, _ = ops.weights_shard(K, N, rank, ws)
    # input sets: the same X, W and bias on every GPU (one GEMM split by columns); enough sets that the bytes read
    # between two uses of one set (X, its decoded copy, this GPU's weight bytes) exceed the L2
    per_set = M * K * 2 * 2 + K * ncols * 9 / 8
    nsets = max(3, int(1.5 * L2_BYTES / per_set) + 2)
    sets, W0 = [], None
    for s in range(nsets):
        g = torch.Generator(device=dev)
        g.manual_seed(1234 + s)
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        W = torch.randn((K, N), generator=g, device=dev) * 0.02
        w_full = ops.PackedWeight.from_float(W)
        b = (torch.randn((N,), generator=g, device=dev) * 0.01).to(torch.bfloat16)
        if s == 0:
            W0, w0_full = W, w_full
        del W
        sets.append((x, w_full.shard(rank, ws)[0], b[n0:n0 + ncols].contiguous(), b))
    dq = torch.empty((M, K), dtype=torch.bfloat16, device=dev)
    out = torch.empty((M, ncols), dtype=torch.bfloat16, device=dev)
    gws = ops.gemm_workspace(M, K, ncols, dev, epilogue=L.RL_EPI_BIAS)   # split-K partials, if the shape splits
    gws_ptr, gws_bytes = (0, 0) if gws is None else (gws.data_ptr(), gws.numel())

    # the timed loop calls the C ABI directly on preallocated buffers (no allocation inside a step)
    def quant(x):
        L.call("rl_quantize_bfp16", x.data_ptr(), L.RL_BF16, M, K, L.RL_ROWMAJOR, None, dq.data_ptr(),
               stream.cuda_stream)

    def gemm(w, b):
        L.call("rl_linear_bfp16_ws", dq.data_ptr(), M, K, w.native.data_ptr(), ncols, b.data_ptr(), L.RL_EPI_BIAS,
               out.data_ptr(), L.RL_BF16, gws_ptr, gws_bytes, stream.cuda_stream)

    def step(i, ev=None):  # quantiser + GEMM
        x, w, b, _ = sets[i % nsets]
        quant(x)
        if ev is not None:
            ev[0].record(stream)
        gemm(w, b)
        if ev is not None:
            ev[1].record(stream)

    # parity of the step's GEMM before timing it
    quant(sets[0][0])

    def gemm0():
        gemm(sets[0][1], sets[0][2])
        return out
    equal, sched, err = gemm_parity(dq, W0, sets[0][3], w0_full, sets[0][1], n0, gemm0, stream, ws)
    del W0, w0_full
    torch.cuda.empty_cache()
    worst = _max_over_ranks([0.0 if (equal is None or equal) else 1.0, sched, err], dev, ws)
    parity = {"max_rel_vs_fp32_sampled_rows": worst[2], "rows_checked": 64, "bar": BF16_OUT_TOL,
              "max_rel_vs_unsplit": worst[1], "split_k": gws is not None,
              "sharded_columns_equal_unsharded": (worst[0] == 0.0) if ws > 1 else None}
    parity["ok"] = worst[2] <= BF16_OUT_TOL and worst[1] <= 2.0 ** -8 and worst[0] == 0.0
    failures = [] if parity["ok"] else [f"C1 GEMM parity: {parity}"]

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    ops.device_status()

    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    gemm_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            step(i, gemm_ev[i])
        t1.record(stream)
        torch.cuda.synchronize()
    ms = _max_over_ranks([t0.elapsed_time(t1)], dev, ws)[0]
    gemm_ms = sum(a.elapsed_time(b) for a, b in gemm_ev) / args.steps
    if ws > 1:
        dist.barrier()
    ops.device_status()

    # end to end through the public API with host buffers: pinned X in, quantise + GEMM, this GPU's C columns back to
    # pinned memory, every step. A serving loop keeps the copy engines busy: step i's X comes in on one stream and
    # step i's C goes out on another while the compute stream works on the step between them (two device buffers
    # each for X and C; events order every buffer's reuse), so the loop runs at the rate of its slowest leg - here
    # the 107 MB device-to-host copy of C - instead of the sum of the three.
    xh = [sets[s][0].cpu().pin_memory() for s in range(min(3, nsets))]
    xd = [torch.empty((M, K), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    od = [out, torch.empty((M, ncols), dtype=torch.bfloat16, device=dev)]
    oh = torch.empty((M, ncols), dtype=torch.bfloat16).pin_memory()
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e2e_steps = max(4, min(args.steps, 50))

    def gemm_into(w, b, o):
        L.call("rl_linear_bfp16_ws", dq.data_ptr(), M, K, w.native.data_ptr(), ncols, b.data_ptr(), L.RL_EPI_BIAS,
               o.data_ptr(), L.RL_BF16, gws_ptr, gws_bytes, stream.cuda_stream)

    def e2e_loop(n, start):
        done_cmp = [None, None]
        done_out = [None, None]
        for i in range(n):
            j = i % 2
            s_in.wait_event(start)
            if done_cmp[j] is not None:
                s_in.wait_event(done_cmp[j])        # the compute of step i - 2 has read xd[j]
            with torch.cuda.stream(s_in):
                xd[j].copy_(xh[i % len(xh)], non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
            stream.wait_event(ev_in)
            if done_out[j] is not None:
                stream.wait_event(done_out[j])      # the copy-out of step i - 2 has read od[j]
            quant(xd[j])
            _, w, b, _ = sets[i % nsets]
            gemm_into(w, b, od[j])
            done_cmp[j] = torch.cuda.Event()
            done_cmp[j].record(stream)
            s_out.wait_event(done_cmp[j])
            with torch.cuda.stream(s_out):
                oh.copy_(od[j], non_blocking=True)
            done_out[j] = torch.cuda.Event()
            done_out[j].record(s_out)
        stream.wait_event(done_out[(n - 1) % 2])
        stream.wait_event(done_cmp[(n - 1) % 2])

    s0 = torch.cuda.Event()
    s0.record(stream)
    e2e_loop(3, s0)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_loop(e2e_steps, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks([e0.elapsed_time(e1)], dev, ws)[0]
    del xh, xd, oh, od

    extras = {}
    if not args.no_extras:
        # the other configs run right after the timed loop; their SM clock is sampled too (after the GEMM loop has
        # reached the power cap the clock stays lowered for a while)
        with ClockSampler(local) as clk_x:
            extras, f2 = measure_configs(dev, stream, ws, rank)
        failures += f2
        extras["clocks"] = clk_x.summary()
        extras["device"] = {"sms": torch.cuda.get_device_properties(dev).multi_processor_count,
                            "pair_gemm_clusters": L.lib().rl_gemm_pair_clusters()}
        for key in ("C2_swiglu_mlp", "C3_joint_attention_sublayer", "C4_dit_step"):
            e = extras[key]
            mx = _max_over_ranks([e["ms"]], dev, ws)[0]
            e["TFLOP/s"] *= e["ms"] / mx
            e["ms"] = mx
        extras["note"] = ("C2, C3, C4 and next_rows: per-GPU timings (each GPU its own copy; max over ranks); C5 GEMM "
                          "sweep: one GEMM split by weight columns over the GPUs; C4 TP: one step split over the GPUs")

    if rank != 0:
        if ws > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    pk, pk_kind = peaks()
    clocks = clk.summary()
    # a GEMM timed over a long loop runs under the power cap: compare it with the measured sustained peak when the
    # sampled clocks show the cap, with the burst peak otherwise (both fractions are reported)
    capped = "sw_power_cap" in clocks.get("reasons", [])
    peak = pk["bf16_tflops_sustained"] if capped else pk["bf16_tflops"]
    launch_flop = 2.0 * M * ncols * K
    achieved = launch_flop / (gemm_ms * 1e-3) / 1e12
    value = FLOP * args.steps / (ms * 1e-3) / 1e12
    res = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
           "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N, "global_batch": 1,
                      "parallelism": (f"N-split over {ws} GPUs: GPU g streams weight columns [g*{ncols}, (g+1)*{ncols})"
                                      f" in place and writes C[:, those columns]; X quantised on every GPU; no "
                                      f"collective" if ws > 1 else "1 GPU"),
                      "columns_per_gpu": ncols,
                      "l2": f"inputs rotate over {nsets} sets ({per_set / 1e6:.0f} MB read per set per GPU) > the "
                            f"126 MB L2"},
           "parity": parity,
           "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak,
                        "traffic": ncu_traffic() if ws == 1 else None,
                        "kernel": "bfp16_linear_pair_kernel",
                        "peak_kind": f"{pk_kind} bf16 dense ({'sustained, power cap seen' if capped else 'burst'})",
                        "frac_of_burst_peak": achieved / pk["bf16_tflops"],
                        "frac_of_sustained_peak": achieved / pk["bf16_tflops_sustained"],
                        "algorithmic_flop_per_launch": launch_flop,
                        "launch_ms": gemm_ms},
           "clocks": clocks,
           "e2e": {"value": FLOP * e2e_steps / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                   "h2d_bytes_per_step": M * K * 2 * ws, "d2h_bytes_per_step": M * N * 2,
                   "note": "pinned host X in and this GPU's C columns out every step, on their own streams so that "
                           "step i's copies overlap the compute of the step between them; bound by the device-to-host "
                           "copy (the bf16 C is 107 MB per step)"},
           "gpu_launches": 2 * args.steps,
           "configs": extras,
           "kernel_ms": {"bfp16_linear": gemm_ms, "quantize+linear": ms / args.steps}}
    if ws > 1:
        res["roofline"]["traffic_note"] = ("no ncu capture of the column-split launch (its X reads do not shrink with "
                                           "the split, so the 1-GPU capture does not scale)")
    if ws == 1 and not args.no_cpu_baseline:
        tf, dt, cores = cpu_baseline_sample()
        res["cpu_baseline"] = {"value": tf, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                               "sample": f"config 1 in full ({M} rows) once: to_bfp16(a_layout) + from_bfp16 + "
                                         f"float32 matmul with bias, numpy/OpenBLAS on {cores} threads, {dt:.2f} s"}
        if not args.no_extras:
            bt, bcores = cpu_dit_block_sample()
            c4 = {"one_block_s": bt, "step_estimate_ms": 32e3 * bt, "cores": bcores,
                  "sample": "config 4's shapes with one block (embedding + block + projection), the CPU oracle of "
                            "the block math once; the 32-block step estimated as 32 x that"}
            gpu_ms = extras.get("C4_dit_step", {}).get("ms")
            if gpu_ms:
                c4["gpu_step_ms"] = gpu_ms
                c4["gpu_speedup"] = 32e3 * bt / gpu_ms
            res["cpu_baseline"]["c4_dit_step"] = c4
    res["parity_ok"] = not failures
    if failures:
        res["parity_failures"] = failures
    print(json.dumps(res), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if failures:
        sys.stderr.write("PARITY FAILED: " + "; ".join(failures) + "\n")
    # the measured GEMM itself must match; the configs' checks are reported in the line (parity_ok / failures)
    return 0 if parity["ok"] else 1


# ------------------------------------------------------------------------------------------------------------------
# profiling cases: one kernel (or one DiT block) on its benchmark-config shape, the target of ncu captures
# ------------------------------------------------------------------------------------------------------------------

CASES = ("linear_c1", "quantize_c1", "linear_m17408", "swiglu_mlp_c2", "swiglu_up_c2", "attention_c3", "qkv_post_c3",
         "qkv_gemm_c4", "qkv_linear_c4", "ln_mod_c4", "dit_block_c4", "vae_conv_128x1152", "vae_conv_512x288",
         "scatter_gemm_tp2", "ln_rows_tp2")


def run_case(case, iters):
    """Inputs are seeded synthetic tensors of the configs' shapes (a few hundred MB on the device at most)."""
    import torch
    from redline_tiny_b200 import _lib as L
    from redline_tiny_b200 import dit, ops
    if case not in CASES:
        raise SystemExit(f"unknown case {case}; cases: {', '.join(CASES)}")
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    s = torch.cuda.current_stream().cuda_stream
    c = case
    if c in ("linear_c1", "quantize_c1", "linear_m17408"):
        Mc, Kc, Nc = (17408 if c == "linear_m17408" else 4352), 3072, 12288
        x = torch.randn((Mc, Kc), generator=g, device=dev).to(torch.bfloat16)
        dq = torch.empty_like(x)
        w = ops.PackedWeight.from_float(torch.randn((Kc, Nc), generator=g, device=dev) * 0.02)
        out = torch.empty((Mc, Nc), dtype=torch.bfloat16, device=dev)

        def fn():
            L.call("rl_quantize_bfp16", x.data_ptr(), L.RL_BF16, Mc, Kc, L.RL_ROWMAJOR, None, dq.data_ptr(), s)
            if c != "quantize_c1":
                L.call("rl_linear_bfp16", dq.data_ptr(), Mc, Kc, w.native.data_ptr(), Nc, None, L.RL_EPI_NONE,
                       out.data_ptr(), L.RL_BF16, s)
    elif c in ("swiglu_up_c2", "swiglu_mlp_c2"):
        Mc, Kc, F = 512, 4096, 12288
        x = ops.quantize_bfp16(torch.randn((Mc, Kc), generator=g, device=dev), want_bytes=False)[1]
        w = ops.PackedWeight.from_float(torch.randn((Kc, 2 * F), generator=g, device=dev) * 0.02, swiglu=True)
        wd = ops.PackedWeight.from_float(torch.randn((F, Kc), generator=g, device=dev) * 0.02)
        h = torch.empty((Mc, F), dtype=torch.bfloat16, device=dev)
        o = torch.empty((Mc, Kc), dtype=torch.bfloat16, device=dev)
        wsp = torch.empty(L.lib().rl_swiglu_mlp_workspace(Mc, Kc, F, 0), dtype=torch.uint8, device=dev)

        def fn():
            if c == "swiglu_up_c2":
                ops.swiglu_up(x, w, out=h)
            else:
                ops.swiglu_mlp(x, w, wd, out=o, workspace=wsp)
    elif c in ("scatter_gemm_tp2", "ln_rows_tp2"):
        # the peer reduce-scatter's two kernels at TP-2 shapes, with both "ranks'" buffers on this GPU: the out
        # projection of 12 heads scattering its partial rows (K 1536), and the row-sharded LayerNorm over 2176 rows
        # adding two partials and storing its rows into two A operands (the wait is satisfied before the launch)
        Mc, D = 4352, 3072
        R = Mc // 2
        if c == "scatter_gemm_tp2":
            Kc = 1536
            x = ops.quantize_bfp16(torch.randn((Mc, Kc), generator=g, device=dev), want_bytes=False)[1]
            w = ops.PackedWeight.from_float(torch.randn((Kc, D), generator=g, device=dev) * 0.02)
            bufs = [torch.empty(R * D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            dsts = torch.tensor([t.data_ptr() for t in bufs], dtype=torch.int64, device=dev)

            def fn():
                L.call("rl_linear_bfp16_scatter", x.data_ptr(), Mc, Kc, w.native.data_ptr(), D, dsts.data_ptr(), 2, R,
                       s)
        else:
            xin = torch.randn((R, D), generator=g, device=dev).to(torch.bfloat16)
            parts = [torch.randn((R * D,), generator=g, device=dev).to(torch.bfloat16) for _ in range(2)]
            parts_t = torch.tensor([t.data_ptr() for t in parts], dtype=torch.int64, device=dev)
            pad = torch.tensor([1 << 40, 0], dtype=torch.int64, device=dev)   # rank 1 sees rank 0's epoch
            params = (1 + 0.1 * torch.randn((2, 2, D), generator=g, device=dev)).to(torch.bfloat16)
            xo = torch.empty((R, D), dtype=torch.bfloat16, device=dev)
            outs = [torch.empty((Mc, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
            y_dsts = torch.tensor([t[R:].data_ptr() for t in outs], dtype=torch.int64, device=dev)

            def fn():
                L.call("rl_ln_mod_tp_rs", xin.data_ptr(), parts_t.data_ptr(), 2, pad.data_ptr(), 1, 1,
                       params.data_ptr(), R, D, 0, xo.data_ptr(), y_dsts.data_ptr(), s)
    elif c in ("vae_conv_128x1152", "vae_conv_512x288"):
        H, C = (128, 1152) if c == "vae_conv_128x1152" else (512, 288)
        x = ops.quantize_bfp16(torch.randn((H * H, C), generator=g, device=dev), want_bytes=False)[1].view(H, H, C)
        pw, bias, taps = ops.conv_weight(torch.randn((C, C, 3, 3), generator=g, device=dev) * 0.02,
                                         torch.randn(C, generator=g, device=dev) * 0.01)
        y = torch.empty((H, H, pw.N), dtype=torch.bfloat16, device=dev)

        def fn():
            ops.conv2d(x, pw, bias, taps, out=y)
    else:
        cfg = dit.DiTConfig(blocks=1)
        model = dit.DiT(cfg, dit.random_weights(cfg, seed=0))
        model.set_t(0.5)
        model.embed(torch.randn((cfg.image, cfg.latent_ch), generator=g, device=dev),
                    torch.randn((cfg.text, cfg.hidden), generator=g, device=dev))
        b = model.blocks[0]
        model._linear(model.a, b["qkv"], model.qkv)

        def qkv_post():
            L.call("rl_qkv_post", model.qkv.data_ptr(), model.rope_cs.data_ptr(), b["wq"].data_ptr(),
                   b["wk"].data_ptr(), cfg.M, cfg.heads, model.q.data_ptr(), model.k.data_ptr(), model.vt.data_ptr(),
                   model.ldv, s)
        qkv_post()

        def attention():
            L.call("rl_attention", model.q.data_ptr(), model.k.data_ptr(), model.vt.data_ptr(), model.ldv, cfg.heads,
                   cfg.M, cfg.M, cfg.M, None, 1.0, model.o.data_ptr(), cfg.hidden, s)
        attention()
        model._linear(model.o, b["o"], model.c)
        def qkv_linear():
            L.call("rl_qkv_linear", model.a.data_ptr(), cfg.M, cfg.hidden, b["qkv"].native.data_ptr(), cfg.heads,
                   cfg.heads, model.rope_cs.data_ptr(), b["wq"].data_ptr(), b["wk"].data_ptr(), model.q.data_ptr(),
                   model.k.data_ptr(), model.vt.data_ptr(), model.ldv, s)
        fn = {"attention_c3": attention, "qkv_post_c3": qkv_post, "qkv_linear_c4": qkv_linear,
              "qkv_gemm_c4": lambda: model._linear(model.a, b["qkv"], model.qkv),
              "ln_mod_c4": lambda: model._ln(model.x[0], model.c, model.params["mlp"], model.x[1], model.a),
              "dit_block_c4": lambda: model.block(0)}[c]
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    t = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    print(f"{c}: last call {1e3 * (time.perf_counter() - t):.3f} ms wall", flush=True)
    L.device_status()
    return 0


def main():
    args = parse()
    if args.case:
        return run_case(args.case, args.iters)
    if args.impl == "reference":
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return 0
    ws, rank, local = dist_init()
    return run_ours(args, ws, rank, local)


if __name__ == "__main__":
    sys.exit(main())
