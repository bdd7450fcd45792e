"""Benchmark of the kebab-b200 GEMM path (one JSON line on rank 0).

Workload (M=N=K=8192 FP16 RC, N(0,1)/sqrt(K) inputs),
M-sharded across ranks with WEAK scaling: every rank owns an 8192-row block
of A (global M = 8192 * world), B (8192 x 8192, column-major) is broadcast
once from rank 0 over NCCL before timing (the broadcast is timed on its own
and reported as `broadcast_ms`), and each rank writes its own column-major C
shard. A step is one kebab_gemm launch per rank. With N=1 this is exactly the
single-GPU 8192^3 headline.

Timing: W warm-up steps, then K timed steps between a barrier + synchronize
on both sides, one CUDA event pair on the launching stream around the K
back-to-back launches (consecutive launches overlap prologue and tail through
programmatic dependent launch; an event between them would serialise them),
max over ranks. Three
rotating input sets (3 x 256 MiB of A + B per rank, > 126 MB L2) keep
consecutive steps from hitting inputs left in L2 by the previous step.

`--impl reference` times the reference's own CPU GEMM (referenceGemmCpp
<float> compiled from the reference sources into oracle/_ref, one row block
per host thread) on a bounded sample of the same workload.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP16 RC GEMM TFLOP/s @ M=N=K=8192, % of B200 dense peak; 1/2/4/8-GPU aggregate"
UNIT = "TFLOP/s"
NOMINAL_DENSE_TFLOPS = 2250.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", default="kebab", choices=["kebab", "reference"])
    p.add_argument("--version", type=int, default=120, help="ladder rung (120 = heuristic)")
    # Capitalised flags: under torchrun a lowercase --m is taken as an
    # abbreviation of torchrun's own options.
    p.add_argument("--M", "--m", dest="m", type=int, default=8192, help="rows of A per rank (global M with --strong)")
    p.add_argument("--strong", action="store_true",
                   help="strong scaling: --M is the global M, row-sharded over the ranks (config 3: "
                        "--strong --M 32768 --N 32768 --K 32768 --dtype bf16)")
    p.add_argument("--N", "--n", dest="n", type=int, default=8192)
    p.add_argument("--K", "--k", dest="k", type=int, default=8192)
    p.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"])
    p.add_argument("--workload", default="dense", choices=["dense", "sparse24"],
                   help="dense GEMM (BASELINE config 2) or 2:4 sparse GEMM (config 5)")
    p.add_argument("--e2e-steps", type=int, default=20)
    p.add_argument("--bcast-chunks", type=int, default=4,
                   help="N-chunks of the pipelined broadcast + GEMM measurement (N > 1 GPUs)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-cublas", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the other BASELINE configs (C2 2048/4096, C4a, C4b, C5 at N=1; C3 strong and C4a "
                        "at every N); they run by default with the default headline workload")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU work for the cpu_baseline sample")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"bf16_tflops": float(d["bf16_tflops"]), "bf16_tflops_sustained": float(d["bf16_tflops_sustained"]),
                "hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def load_traffic(workload):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            d = json.load(f)
        return d.get(workload)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
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
        self.thread.join(timeout=2)
        sms, maxes, watts, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            try:
                watts.append(float(parts[3].split()[0]))
            except (ValueError, IndexError):
                pass
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sms:
            return None
        out = {"sm_mhz": float(np.median(sms)), "sm_max_mhz": float(max(maxes)), "reasons": sorted(reasons),
               "samples": len(sms)}
        if watts:
            out["power_w"] = float(np.median(watts))
        return out


def kb_sm_count(torch, local):
    return torch.cuda.get_device_properties(local).multi_processor_count


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def make_inputs(torch, M, N, K, dtype, device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    s = 1.0 / np.sqrt(K)
    A = (torch.randn((M, K), generator=g, device=device, dtype=torch.float32) * s).to(dtype)
    B = (torch.randn((N, K), generator=g, device=device, dtype=torch.float32) * s).to(dtype)
    return A, B


def cpu_model():
    """The host CPU's model name (first `model name` line of /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_reference_1core(M, N, K, n=512):
    """referenceGemmCpp<float> as the reference ships it (single thread,
    compiled from its own header into oracle/_ref) at n^3 on the C1 inputs
    (mt19937(0) uniform[-1, 1], FP16), with the time it would take for the
    full M x N x K workload extrapolated from its rate. Falls back to the
    restatement on one thread when oracle/_ref is not built."""
    import oracle as O
    A, B = O.fill_pair(n, n, n, seed=0, dtype=O.F16, dist=O.UNIFORM)
    L = O.ref()
    if L is not None:
        Af = np.ascontiguousarray(O.to_float(A, O.F16), np.float32)
        Bf = np.ascontiguousarray(O.to_float(B, O.F16), np.float32)
        C = np.empty(n * n, np.float32)
        t0 = time.perf_counter()
        L.kbr_gemm_f32(Af, Bf, C, n, n, n)
        dt = time.perf_counter() - t0
        kind = "reference"
    else:
        t0 = time.perf_counter()
        O.gemm(A, B, n, n, n, O.F16, threads=1)
        dt = time.perf_counter() - t0
        kind = "port"
    gflops = 2.0 * n ** 3 / dt / 1e9
    return {"gflops": gflops, "cores": 1, "kind": kind, "size": "%d^3" % n, "seconds": dt,
            "extrapolated_s_full_workload": 2.0 * M * N * K / (gflops * 1e9)}


def cpu_baseline_port(M, N, K, target_s):
    """The oracle restatement (bit-identical to referenceGemmCpp<float>) on all
    host cores over a bounded row sample of the workload."""
    import oracle as O
    threads = cpu_threads()
    A, B = O.fill_pair(min(M, 256), N, K, seed=0, dtype=O.F16, dist=O.NORMAL, scale_a=1 / np.sqrt(K),
                       scale_b=1 / np.sqrt(K))
    Mp = min(M, 256)
    rows = np.arange(0, min(Mp, threads), dtype=np.int64)
    t0 = time.perf_counter()
    O.gemm_rows(A, B, rows, Mp, N, K, O.F16, threads)
    dt = time.perf_counter() - t0
    # Enough rows for about target_s of CPU work; rows cycle over the Mp
    # generated ones (each row reads all of B, so repeats cost the same).
    n_rows = len(rows)
    for _ in range(3):  # the first timings include thread start-up: refine twice
        n_rows = int(max(n_rows, min(64 * Mp, round(n_rows * target_s / max(dt, 1e-3)))))
        rows = np.arange(n_rows, dtype=np.int64) % Mp
        t0 = time.perf_counter()
        O.gemm_rows(A, B, rows, Mp, N, K, O.F16, threads)
        dt = time.perf_counter() - t0
        if dt >= 0.9 * target_s or n_rows >= 64 * Mp:
            break
    flops = 2.0 * n_rows * N * K
    return {"value": flops / dt / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": "%d rows x %d cols of C (K=%d) of the %dx%dx%d workload, %.1f s" % (n_rows, N, K, M, N, K, dt)}


class RefCpuGemm:
    """referenceGemmCpp<float> (compiled from the reference sources into
    oracle/_ref) over row blocks, one block per host thread."""

    def __init__(self, N, K, threads, rows_per_thread):
        import oracle as O
        self.L = O.ref()
        if self.L is None:
            raise RuntimeError("oracle/_ref/libkebab_ref.so not built")
        self.N, self.K, self.threads, self.rpt = N, K, threads, rows_per_thread
        rows = threads * rows_per_thread
        A, B = O.fill_pair(rows, N, K, seed=0, dtype=O.F16, dist=O.NORMAL, scale_a=1 / np.sqrt(K),
                           scale_b=1 / np.sqrt(K))
        self.A = O.to_float(A, O.F16).reshape(rows, K)
        self.B = np.ascontiguousarray(O.to_float(B, O.F16))
        self.C = [np.empty(rows_per_thread * N, np.float32) for _ in range(threads)]

    def step(self):
        def work(t):
            a = np.ascontiguousarray(self.A[t * self.rpt:(t + 1) * self.rpt].reshape(-1))
            self.L.kbr_gemm_f32(a, self.B, self.C[t], self.rpt, self.N, self.K)
        ts = [threading.Thread(target=work, args=(t,)) for t in range(self.threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        return 2.0 * self.threads * self.rpt * self.N * self.K


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = cpu_threads()
    M, N, K = args.m, args.n, args.k
    workload = "gemm_rc_%s_%dx%dx%d_msharded" % (args.dtype, M, N, K)
    try:
        ref = RefCpuGemm(N, K, threads, 1)
    except Exception as e:
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU GEMM not built: %s" % e}))
        return
    # Size one step at ~2 s of CPU work so warm-up + steps stay within minutes.
    t0 = time.perf_counter()
    ref.step()
    dt1 = time.perf_counter() - t0
    rpt = max(1, min(64, int(2.0 / max(dt1, 1e-3))))
    ref = RefCpuGemm(N, K, threads, rpt)
    for _ in range(args.warmup):
        ref.step()
    t0 = time.perf_counter()
    flops = 0.0
    for _ in range(args.steps):
        flops += ref.step()
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    sample = ("referenceGemmCpp<float> (reference source, compiled -O3 -ffp-contract=off), %d threads x %d rows "
              "x %d cols of C per step (K=%d) of the %dx%dx%d workload" % (threads, rpt, N, K, M, N, K))
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (fp16 inputs widened)", "data": "synthetic",
        "config": {"workload": workload, "M_per_rank": M, "N": N, "K": K, "layout": "RC", "threads": threads},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ----------------------------------------------------------------------------
# Per-config extras: the other BASELINE configurations, each timed on the
# device (one event pair around back-to-back launches, max over ranks), with a
# sampled check of this rank's output against the CPU oracle outside the
# timed region, the SM clock of the last timed launch read from the kernel's
# own clock probe, and cuBLAS in the same loop on rank 0 at N = 1.
# ----------------------------------------------------------------------------
DENSE_FLOP_PER_CLK_SM = 8192.0  # tcgen05 kind::f16, measured (microbench)


def _round_bf16(c):
    u = np.asarray(c, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def sample_parity(torch, A, B, C, bf16, seed, rows=3, row_cols=1024, elems=4096, threads=1):
    """Checks a seeded sample of C ([N, M] column-major tensor = A [M, K] * B
    [N, K]^T) against the oracle restatement of the reference CPU GEMM: the
    first, the last and one random row over `row_cols` consecutive columns,
    plus `elems` random elements. Tolerance: relative Frobenius <= 1e-3 and
    |d| <= 1e-2 (1 + |ref|) per element; for BF16 output against the oracle
    rounded to BF16, with the raw distance to the FP32 oracle under 4e-3."""
    import oracle as O
    M, K = A.shape
    N = B.shape[0]
    g = np.random.default_rng(seed)
    rs = np.unique(np.array([0, M - 1, int(g.integers(0, M))]))[:rows]
    c0 = int(g.integers(0, max(1, N - row_cols + 1)))
    cols = np.arange(c0, min(N, c0 + row_cols))
    ii = np.concatenate([g.integers(0, M, elems), np.repeat(rs, cols.size)]).astype(np.int64)
    jj = np.concatenate([g.integers(0, N, elems), np.tile(cols, rs.size)]).astype(np.int64)
    ur, ir = np.unique(ii, return_inverse=True)
    uc, ic = np.unique(jj, return_inverse=True)
    dev = A.device

    def bits(t, idx):
        sub = t[torch.from_numpy(idx).to(dev)].contiguous()
        return sub.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)

    Ah, Bh = bits(A, ur), bits(B, uc)
    got = C[torch.from_numpy(jj).to(dev), torch.from_numpy(ii).to(dev)].float().cpu().numpy()
    dt = O.BF16 if bf16 else O.F16
    want = O.gemm_elems(Ah, Bh, ir.astype(np.int64), ic.astype(np.int64), ur.size, uc.size, K, dt, threads)
    out = {"elements": int(ii.size)}
    ok = True
    if bf16:
        ok_raw, rel_raw, _ = O.check_tolerance(got, want, 4e-3, 1e-2)
        out["rel_fro_raw"] = rel_raw
        ok = ok and ok_raw
        want = _round_bf16(want)
    ok2, rel, worst = O.check_tolerance(got, want, 1e-3, 1e-2)
    out.update({"ok": bool(ok and ok2), "rel_fro": rel, "worst_elem_ratio": worst})
    return out


class Extras:
    def __init__(self, torch, dist, kb, rank, world, device, stream, sm_count, cublas):
        self.torch, self.dist, self.kb = torch, dist, kb
        self.rank, self.world, self.device, self.stream = rank, world, device, stream
        self.sm_count = sm_count
        self.cublas = cublas and rank == 0 and world == 1
        self.threads = max(1, cpu_threads() // max(1, world))

    def sync(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device=self.device, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_true(self, ok):
        if self.world == 1:
            return bool(ok)
        t = self.torch.tensor([0.0 if ok else 1.0], device=self.device, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.item() == 0.0

    def loop_ms(self, fn, steps, warmup, probe=True):
        """Device ms of `steps` back-to-back calls (one event pair, max over
        ranks) and the time-weighted SM clock of all of them (clock probe)."""
        torch = self.torch
        for i in range(warmup):
            fn(i)
        probe_buf = torch.zeros((steps, 256, 4), dtype=torch.int64, device=self.device) if probe else None
        self.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for i in range(steps):
            if probe:
                self.kb.clock_probe(probe_buf[i])  # each launch records its own SM clock
            fn(i)
        e1.record(self.stream)
        torch.cuda.synchronize()
        self.kb.clock_probe(None)
        rc, code = self.kb.device_status()
        if rc != self.kb.OK:
            raise RuntimeError("device status 0x%x" % code)
        ms = self.max_over_ranks(e0.elapsed_time(e1))
        clk = self.kb.clock_probe_mhz(probe_buf) if probe else None
        return ms, clk

    def cublas_ms(self, As, Bs, steps, warmup):
        torch = self.torch
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        n = len(As)
        for i in range(warmup):
            torch.matmul(As[i % n], Bs[i % n].t())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for i in range(steps):
            torch.matmul(As[i % n], Bs[i % n].t())
        e1.record(self.stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    def inputs(self, M, N, K, dtype, seed, a_std=None, b_std=None):
        torch = self.torch
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        a_std = 1.0 / np.sqrt(K) if a_std is None else a_std
        b_std = 1.0 / np.sqrt(K) if b_std is None else b_std
        A = torch.empty((M, K), dtype=dtype, device=self.device)
        B = torch.empty((N, K), dtype=dtype, device=self.device)
        for T, std in ((A, a_std), (B, b_std)):  # in row slabs: no 4-byte temporary of the whole operand
            step = max(1, (1 << 28) // (4 * K))
            for r0 in range(0, T.shape[0], step):
                r1 = min(T.shape[0], r0 + step)
                T[r0:r1] = (torch.randn((r1 - r0, K), generator=g, device=self.device) * std).to(dtype)
        return A, B

    def clock_fields(self, tflops, clk, sparse=False):
        if not clk:
            return {}
        peak = self.sm_count * DENSE_FLOP_PER_CLK_SM * (2.0 if sparse else 1.0) * clk["sm_mhz"] * 1e6 / 1e12
        return {"effective_sm_mhz": clk["sm_mhz"], "frac_of_clock_peak": tflops / peak,
                "clock_peak_tflops": peak, "probe": clk}

    def dense(self, name, M_global, N, K, bf16, sets, steps, warmup, version=120, a_std=None, b_std=None,
              sharded=True, bcast_b=False):
        """A dense config, M-sharded over the ranks (rank r owns a row block);
        with bcast_b, B of the first input set is broadcast from rank 0 first,
        so every rank multiplies by the same B."""
        torch, kb = self.torch, self.kb
        dtype = torch.bfloat16 if bf16 else torch.float16
        code = kb.BF16 if bf16 else kb.F16
        M = M_global // self.world if sharded else M_global
        data = []
        for s in range(sets):
            A, B = self.inputs(M, N, K, dtype, 7919 * s + 31 * self.rank + M_global, a_std, b_std)
            data.append((A, B, torch.empty((N, M), dtype=dtype, device=self.device)))
        if bcast_b and self.world > 1:
            self.dist.broadcast(data[0][1], src=0)  # also sets up NCCL for the large broadcasts below
            self.sync()
        sp = self.stream.cuda_stream

        def step(i):
            A, B, C = data[i % sets]
            rc = kb.gemm_raw(code, A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, "RC", version, sp)
            if rc != kb.OK:
                raise kb.KebabError(rc, kb.last_error())

        ms, clk = self.loop_ms(step, steps, warmup)
        per = ms / steps
        flops = 2.0 * M_global * N * K if sharded else 2.0 * M * N * K * self.world
        tflops = flops / (per * 1e-3) / 1e12
        rung = kb.lib().kebab_resolve_version(version, code, M, N, K)
        out = {"workload": name, "M": M_global, "N": N, "K": K, "M_per_rank": M, "dtype": "bf16" if bf16 else "fp16",
               "rung": rung, "rung_name": kb.version_name(rung), "launches": steps, "input_sets": sets,
               "ms_per_gemm": per, "tflops": tflops}
        out.update(self.clock_fields(tflops / self.world, clk))
        if self.cublas:
            cb = self.cublas_ms([d[0] for d in data], [d[1] for d in data], steps, warmup)
            out["cublas_tflops"] = 2.0 * M * N * K / (cb * 1e-3) / 1e12
            out["vs_cublas"] = tflops / out["cublas_tflops"]
        A, B, C = data[0]
        step(0)
        torch.cuda.synchronize()
        par = sample_parity(torch, A, B, C, bf16, seed=M_global + N + self.rank, threads=self.threads)
        out["parity"] = par
        out["parity_all_ranks"] = self.all_true(par["ok"])
        return out, data

    def hbm(self, out, M, N, K):
        """Roofline of an HBM-bound config: algorithmic bytes (A + B read, C
        written once) over the measured launch time."""
        nbytes = 2.0 * (M * K + N * K + M * N)
        gbs = nbytes / (out["ms_per_gemm"] * 1e-3) / 1e9
        peaks = load_peaks()
        out.update({"algorithmic_bytes": nbytes, "gbs": gbs, "hbm_peak_gbs": peaks["hbm_gbs"],
                    "frac_of_hbm": gbs / peaks["hbm_gbs"], "frac_of_8tbs": gbs / 8000.0})
        if "cublas_tflops" in out:
            out["cublas_gbs"] = nbytes / (2.0 * M * N * K / (out["cublas_tflops"] * 1e12)) / 1e9
        return out

    def c3_strong(self, steps=5, warmup=2):
        """32768^3 BF16 split into M row blocks; B (2 GiB)
        broadcast from rank 0. GEMM-only time, the broadcast alone, and
        broadcast followed by the GEMM, each device-timed, max over ranks."""
        torch, dist = self.torch, self.dist
        S = 32768
        out, data = self.dense("c3_strong_bf16_32768", S, S, S, True, 1, steps, warmup, bcast_b=True)
        A, B, C = data[0]
        out["scaling"] = "strong"
        if self.world > 1:

            def one(with_gemm):
                self.sync()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
                dist.broadcast(B, src=0)
                if with_gemm:
                    self.kb.gemm(A, B, C, version=120, stream=self.stream)
                e1.record(self.stream)
                torch.cuda.synchronize()
                return self.max_over_ranks(e0.elapsed_time(e1))

            out["broadcast_ms"] = sorted(one(False) for _ in range(3))[1]
            out["broadcast_gbs"] = 2.0 * S * S / (out["broadcast_ms"] * 1e-3) / 1e9
            out["broadcast_plus_gemm_ms"] = sorted(one(True) for _ in range(3))[1]
            out["broadcast_plus_gemm_tflops"] = 2.0 * S ** 3 / (out["broadcast_plus_gemm_ms"] * 1e-3) / 1e12
            cols = int(os.environ.get("KEBAB_BENCH_CHAIN_COLS", "0")) or 1024
            out["overlapped"] = self.chained(A, B, C, chunk_cols=cols, flops=2.0 * S ** 3, mode="push")
            out["overlapped_pull"] = self.chained(A, B, C, chunk_cols=cols, flops=2.0 * S ** 3, mode="pull")
        else:
            out["broadcast_ms"] = 0.0
            out["broadcast_plus_gemm_ms"] = out["ms_per_gemm"]
            out["broadcast_plus_gemm_tflops"] = out["tflops"]
        del data
        return out

    def chained(self, A, B, C, chunk_cols, flops, reps=3, mode="push"):
        """Broadcast of B overlapped with the GEMM: copy-engine pulls down the
        rank chain (kebab_ring_pull) feeding each rank's gated GEMM
        (kebab_gemm_gated). Device time from the GEMM's launch to its end,
        max over ranks, median of `reps`; C is compared bit for bit with the
        plain GEMM's (same rung, same schedule, same B)."""
        torch = self.torch
        from kebab_b200.shard import ChainBroadcastGemm
        # The plain GEMM on the B every rank holds now, once after an idle
        # barrier like the chained calls below (same power state).
        plain = torch.empty_like(C)
        singles = []
        for _ in range(3):
            self.sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            self.kb.gemm(A, B, plain, version=120, stream=self.stream)
            e1.record(self.stream)
            torch.cuda.synchronize()
            singles.append(self.max_over_ranks(e0.elapsed_time(e1)))
        chain = ChainBroadcastGemm(B, chunk_cols=chunk_cols, mode=mode)
        times, copies, mine, mine_copy = [], [], [], []
        try:
            for r in range(3):  # B alone down the chain: device time on the copy stream
                self.sync()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
                chain.run(None, None, stream=self.stream)
                e1.record(self.stream)
                torch.cuda.synchronize()
                mine_copy.append(e0.elapsed_time(e1))
                copies.append(self.max_over_ranks(mine_copy[-1]))
            for r in range(reps + 1):  # the first call maps the peer buffer lazily: not timed
                C.fill_(float("nan"))
                self.sync()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
                chain.run(A, C, version=120, stream=self.stream)
                e1.record(self.stream)
                torch.cuda.synchronize()
                rc, code = self.kb.device_status()
                if rc != self.kb.OK:
                    raise RuntimeError("device status 0x%x in the chained broadcast" % code)
                if r:
                    mine.append(e0.elapsed_time(e1))
                    times.append(self.max_over_ranks(mine[-1]))
            same = self.all_true(torch.equal(C.view(torch.int16), plain.view(torch.int16)))
        finally:
            self.sync()
            chain.close()
        ms = sorted(times)[len(times) // 2]
        per_rank = [None] * self.world
        per_rank_copy = [None] * self.world
        if self.world > 1:
            self.dist.all_gather_object(per_rank, sorted(mine)[len(mine) // 2])
            self.dist.all_gather_object(per_rank_copy, sorted(mine_copy)[1])
        copy_ms = sorted(copies)[1]
        return {"mode": mode, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "per_rank_ms": per_rank,
                "per_rank_copy_ms": per_rank_copy,
                "gemm_single_ms": sorted(singles)[1], "copy_only_ms": copy_ms,
                "copy_only_gbs": B.numel() * B.element_size() / (copy_ms * 1e-3) / 1e9,
                "chunk_cols": chunk_cols, "chunks": chain.nchunks,
                "bitexact_vs_plain_gemm": same,
                "what": "B moved down the rank chain by copy engines (CUDA IPC, NVLink; %s) while every rank's gated "
                        "GEMM runs; device time from GEMM launch to GEMM end, max over ranks, median of %d; "
                        "copy_only: the same chain without GEMMs" % (mode, reps)}

    def sparse(self, M, N, K, sets, steps, warmup):
        """A dense N(0,1) pruned 2:4 and compressed once
        (timed separately: packer GB/s), B N(0,1)/sqrt(K); dense-equivalent
        TFLOP/s (2MNK) against 2x the dense clock peak."""
        torch, kb = self.torch, self.kb
        data = []
        packer = None
        for s in range(sets):
            A, B = self.inputs(M, N, K, torch.float16, 104729 * s + 5, a_std=1.0)
            t0, t1, t2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            t0.record(self.stream)
            pr = kb.sparse24_prune(A)
            t1.record(self.stream)
            pk, E = kb.sparse24_compress(pr)
            t2.record(self.stream)
            torch.cuda.synchronize()
            if s == 0:
                mk = M * K
                packer = {"prune_gbs": 4.0 * mk / (t0.elapsed_time(t1) * 1e-3) / 1e9,
                          "compress_gbs": (2.0 * mk + mk + mk / 8.0) / (t1.elapsed_time(t2) * 1e-3) / 1e9,
                          "prune_ms": t0.elapsed_time(t1), "compress_ms": t1.elapsed_time(t2)}
            del A
            data.append((pr, pk, E, B, torch.empty((N, M), dtype=torch.float16, device=self.device)))
        sp = self.stream.cuda_stream

        def step(i):
            pr, pk, E, B, C = data[i % sets]
            rc = kb._sp().kebab_gemm_sparse24(kb.F16, pk.data_ptr(), E.data_ptr(), B.data_ptr(), C.data_ptr(),
                                             M, N, K, sp)
            if rc != kb.OK:
                raise kb.KebabError(rc, kb.last_error())

        ms, clk = self.loop_ms(step, steps, warmup)
        per = ms / steps
        tflops = 2.0 * M * N * K / (per * 1e-3) / 1e12
        tm, tn = kb.sparse24_tile(M, N)
        out = {"workload": "c5_sparse24_fp16_%d" % M, "M": M, "N": N, "K": K, "tile": [tm, tn], "launches": steps,
               "input_sets": sets, "ms_per_gemm": per, "tflops_dense_equivalent": tflops,
               "tflops_useful": tflops / 2.0, "packer": packer}
        peaks = load_peaks()
        out["frac_of_2x_burst_peak"] = tflops / (2.0 * peaks["bf16_tflops"])
        out.update(self.clock_fields(tflops, clk, sparse=True))
        if self.cublas:
            cb = self.cublas_ms([d[0] for d in data], [d[3] for d in data], steps, warmup)
            out["dense_cublas_tflops"] = 2.0 * M * N * K / (cb * 1e-3) / 1e12
        pr, pk, E, B, C = data[0]
        step(0)
        torch.cuda.synchronize()
        out["parity"] = sample_parity(torch, pr, B, C, False, seed=M + 5, threads=self.threads)
        del data
        return out


def run_extras(args, torch, dist, kb, rank, world, device, stream, sm_count):
    ex = Extras(torch, dist, kb, rank, world, device, stream, sm_count, cublas=not args.no_cublas)
    out = {}
    t0 = time.perf_counter()
    if world == 1:
        for n, sets, steps in ((2048, 10, 200), (4096, 3, 100)):
            r, d = ex.dense("c2_fp16_%d" % n, n, n, n, False, sets, steps, 5, sharded=False)
            del d
            out["c2_%d" % n] = r
        r, d = ex.dense("c4b_decode_fp16_64x8192x8192", 64, 8192, 8192, False, 3, 200, 5, a_std=1.0, b_std=0.02,
                        sharded=False)
        del d
        out["c4b"] = ex.hbm(r, 64, 8192, 8192)
        out["c5"] = ex.sparse(8192, 8192, 8192, 3, 100, 5)
        torch.cuda.empty_cache()
    r, d = ex.dense("c4a_prefill_fp16_16384x28672x8192", 16384, 28672, 8192, False, 1, 10, 3, a_std=1.0,
                    b_std=0.02)
    del d
    out["c4a"] = r
    torch.cuda.empty_cache()
    out["c3_strong"] = ex.c3_strong()
    torch.cuda.empty_cache()
    out["extras_wall_s"] = time.perf_counter() - t0
    return out


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import kebab_b200 as kb

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    dtype = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    M, N, K = args.m, args.n, args.k
    M_global = M
    if args.strong:
        from kebab_b200.shard import row_block
        M = row_block(M_global, world, rank).rows
    else:
        M_global = M * world
    version = args.version
    resolved = kb.lib().kebab_resolve_version(version, kb.F16 if args.dtype == "fp16" else kb.BF16, M, N, K)
    if args.workload == "sparse24":
        tm, tn = kb.sparse24_tile(M, N)
        resolved = "sparse24_%s_%dx%d" % ("1cta" if tm == 128 else "cta_pair", tm, tn)
    sparse = args.workload == "sparse24"
    workload = "%s_rc_%s_%dx%dx%d_msharded%s" % ("gemm_sparse24" if sparse else "gemm", args.dtype,
                                                  M_global if args.strong else M, N, K,
                                                  "_strong" if args.strong else "")
    stream = torch.cuda.current_stream()

    # Inputs: A shards are generated per rank; B on rank 0, then broadcast.
    NSETS = 3
    As, Bs, Cs = [], [], []
    for s in range(NSETS):
        A, B = make_inputs(torch, M, N, K, dtype, device, seed=1000 * s + rank)
        As.append(A)
        Bs.append(B)
        Cs.append(torch.empty((N, M), dtype=dtype, device=device))
    bcast_ms = None
    if world > 1:
        # The first large broadcast sets up NCCL's channels and buffers (~18 ms
        # on two B200s): do it once untimed (rank 0's B is unchanged by it).
        dist.broadcast(Bs[0], src=0)
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s in range(NSETS):
            dist.broadcast(Bs[s], src=0)
        e1.record(stream)
        torch.cuda.synchronize()
        bcast_ms = e0.elapsed_time(e1) / NSETS

    packer = None
    if sparse:
        # Config 5: A dense N(0,1) pruned 2:4 and compressed once, outside timing;
        # the prune and compress kernels are timed separately (GB/s).
        Ps, Es = [], []
        for s in range(NSETS):
            As[s] = As[s] * float(np.sqrt(K))  # N(0,1) activations, as config 5 asks
            t0, t1, t2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            t0.record(stream)
            pr = kb.sparse24_prune(As[s])
            t1.record(stream)
            pk, E = kb.sparse24_compress(pr)
            t2.record(stream)
            torch.cuda.synchronize()
            if s == NSETS - 1:
                mk = M * K
                packer = {"prune_gbs": 4.0 * mk / (t0.elapsed_time(t1) * 1e-3) / 1e9,
                          "compress_gbs": (2.0 * mk + mk + mk / 8.0) / (t1.elapsed_time(t2) * 1e-3) / 1e9,
                          "prune_ms": t0.elapsed_time(t1), "compress_ms": t1.elapsed_time(t2)}
            Ps.append(pk)
            Es.append(E)
            As[s] = pr

    def step(i):
        s = i % NSETS
        if sparse:
            rc = kb._sp().kebab_gemm_sparse24(kb.F16 if args.dtype == "fp16" else kb.BF16, Ps[s].data_ptr(),
                                             Es[s].data_ptr(), Bs[s].data_ptr(), Cs[s].data_ptr(), M, N, K,
                                             torch.cuda.current_stream().cuda_stream)
            if rc != kb.OK:
                raise kb.KebabError(rc, kb.last_error())
            return
        rc = kb.gemm_raw(kb.F16 if args.dtype == "fp16" else kb.BF16, As[s].data_ptr(), Bs[s].data_ptr(),
                         Cs[s].data_ptr(), M, N, K, "RC", version, torch.cuda.current_stream().cuda_stream)
        if rc != kb.OK:
            raise kb.KebabError(rc, kb.last_error())

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    rc, code = kb.device_status()
    if rc != kb.OK:
        raise RuntimeError("device status 0x%x after warm-up" % code)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    # One event pair around the K back-to-back steps (as for the cuBLAS
    # comparator below): an event between two launches would stop the next
    # launch's prologue from overlapping the previous kernel (PDL).
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # Every launch records its own SM clock (cycle counter / global timer per
    # CTA): the time-weighted clock of the timed loop, not of its lead-in.
    probe_buf = torch.zeros((args.steps, 256, 4), dtype=torch.int64, device=device)
    e_start.record(stream)
    for i in range(args.steps):
        kb.clock_probe(probe_buf[i])
        step(i)
    e_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    kb.clock_probe(None)
    probe_clk = kb.clock_probe_mhz(probe_buf)
    rc, code = kb.device_status()
    if rc != kb.OK:
        raise RuntimeError("device status 0x%x after timed steps" % code)
    total_ms = e_start.elapsed_time(e_end)
    # Serialised per-launch durations (an event pair around each of a few
    # launches after the timed region), reported beside the throughput.
    n_pl = min(args.steps, 20)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(n_pl + 1)]
    ev[0].record(stream)
    for i in range(n_pl):
        step(i)
        ev[i + 1].record(stream)
    torch.cuda.synchronize()
    per_launch = [ev[i].elapsed_time(ev[i + 1]) for i in range(n_pl)]
    t = torch.tensor([total_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    flops_rank = 2.0 * M * N * K
    value = world * flops_rank * args.steps / (total_ms * 1e-3) / 1e12

    # First-call latency with the broadcast in it (N > 1, dense): broadcast
    # of B then the GEMM, against the pipelined form that broadcasts B in
    # N-chunks and starts each chunk's GEMM as soon as it has arrived. Device
    # time, max over ranks, median of 3.
    bcast_gemm = None
    if world > 1 and not sparse:
        from kebab_b200.shard import broadcast_gemm_pipelined

        def one(pipelined):
            dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            if pipelined:
                broadcast_gemm_pipelined(As[0], Bs[0], Cs[0], chunks=args.bcast_chunks, version=version, stream=stream)
            else:
                dist.broadcast(Bs[0], src=0)
                kb.gemm(As[0], Bs[0], Cs[0], version=version, stream=stream)
            b.record(stream)
            torch.cuda.synchronize()
            tt = torch.tensor([a.elapsed_time(b)], device=device, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            return float(tt.item())

        one(True)  # warm-up of the chunk shapes
        ser = sorted(one(False) for _ in range(3))[1]
        pip = sorted(one(True) for _ in range(3))[1]
        bcast_gemm = {"serial_ms": ser, "pipelined_ms": pip, "chunks": args.bcast_chunks,
                      "what": "broadcast of B + this rank's GEMM, device time, max over ranks, median of 3; "
                              "pipelined = NCCL broadcast in N-chunks, one GEMM per chunk"}
        try:
            ex = Extras(torch, dist, kb, rank, world, device, stream, kb_sm_count(torch, local), cublas=False)
            bcast_gemm["chained"] = ex.chained(As[0], Bs[0], Cs[0], chunk_cols=1024, flops=2.0 * M * N * K)
        except Exception as e:  # reported, never silent
            bcast_gemm["chained"] = {"error": str(e)[:300]}

    # End to end through the public API with host buffers: every step copies
    # its inputs host -> device from pinned memory (A shard; B on rank 0, then
    # the NCCL broadcast), runs the GEMM and reads its C shard back to pinned
    # host memory, all inside the timed region. Consecutive steps are
    # pipelined over a copy-in, a compute and a copy-out stream with two
    # device buffer sets, so step i's copies overlap step i-1's GEMM, as a
    # serving loop would run them.
    src_a = Ps[0] if sparse else As[0]
    hA = src_a.cpu().pin_memory()
    hE = Es[0].cpu().pin_memory() if sparse else None
    hB = Bs[0].cpu().pin_memory() if rank == 0 else None
    hC = [torch.empty((N, M), dtype=dtype).pin_memory() for _ in range(2)]
    dA = [torch.empty_like(src_a) for _ in range(2)]
    dE = [torch.empty_like(Es[0]) for _ in range(2)] if sparse else None
    dB = [torch.empty_like(Bs[0]) for _ in range(2)]
    dC = [torch.empty_like(Cs[0]) for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_comp[b])  # GEMM i-2 has read set b
            dA[b].copy_(hA, non_blocking=True)
            if sparse:
                dE[b].copy_(hE, non_blocking=True)
            if rank == 0:
                dB[b].copy_(hB, non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[b])
            if i >= 2:
                s_comp.wait_event(ev_out[b])  # C of step i-2 has been read out
            if world > 1:
                dist.broadcast(dB[b], src=0)
            if sparse:
                kb.gemm_sparse24(dA[b], dE[b], dB[b], dC[b], stream=s_comp)
            else:
                kb.gemm(dA[b], dB[b], dC[b], version=version, stream=s_comp)
            ev_comp[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[b])
            hC[b].copy_(dC[b], non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(2):  # warm-up
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(s_in)
    for i in range(args.e2e_steps):
        e2e_step(i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_comp)
    f1.record(s_out)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    e2e_value = world * flops_rank * args.e2e_steps / (e2e_ms * 1e-3) / 1e12
    hC = hC[(args.e2e_steps - 1) % 2]
    h2d = (M * K + N * K) * 2 if not sparse else M * K + N * K * 2 + M * K // 8
    ok_e2e = bool(torch.isfinite(hC.float()).all().item())

    cublas = None
    if not args.no_cublas and rank == 0:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        for _ in range(3):
            torch.matmul(As[0], Bs[0].t())
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_cb = args.steps  # same loop length as the timed region (same power state)
        cb_sampler = ClockSampler(local)
        cb_sampler.start()
        time.sleep(0.3)
        c0.record(stream)
        for i in range(n_cb):
            torch.matmul(As[i % NSETS], Bs[i % NSETS].t())
        c1.record(stream)
        torch.cuda.synchronize()
        cb_clocks = cb_sampler.stop()
        cublas = {"value": flops_rank * n_cb / (c0.elapsed_time(c1) * 1e-3) / 1e12, "unit": UNIT, "clocks": cb_clocks,
                  "what": "torch.matmul (cuBLAS, FP32 accumulate) on the same inputs, 1 GPU, same number of back-to-back launches"}

    # Headline parity: a seeded sample of this rank's C (input set 0) against
    # the oracle, outside every timed region; verdicts gathered over ranks.
    hp = sample_parity(torch, As[0], Bs[0], Cs[0], args.dtype == "bf16", seed=4242 + rank,
                       threads=max(1, cpu_threads() // world))
    t_ok = torch.tensor([0.0 if hp["ok"] else 1.0, hp["rel_fro"], hp["worst_elem_ratio"]], device=device,
                        dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_ok, op=dist.ReduceOp.MAX)
    parity = {"ok": t_ok[0].item() == 0.0, "rel_fro_max": t_ok[1].item(), "worst_elem_ratio_max": t_ok[2].item(),
              "elements_per_rank": hp["elements"], "ranks": world,
              "what": "first, last and one random row x 1024 columns plus 4096 random elements of each rank's C, "
                      "against the oracle restatement of referenceGemmCpp<float>"}

    extras = None
    default_workload = (not args.strong and not sparse and (args.m, args.n, args.k) == (8192, 8192, 8192)
                        and args.dtype == "fp16" and version == 120)
    if default_workload and not args.no_extras:
        del As, Bs, Cs, dA, dB, dC, hA, hB, hC, src_a
        torch.cuda.empty_cache()
        extras = run_extras(args, torch, dist, kb, rank, world, device, stream, kb_sm_count(torch, local))

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks = load_peaks()
    # Average duration of one launch over the timed region (on the launch stream).
    avg_launch_ms = total_ms / args.steps
    achieved = flops_rank / (avg_launch_ms * 1e-3) / 1e12
    # The burst peak was measured at full clock, the sustained one under the
    # power cap: a loop whose sampled SM clock sat below 90 % of the maximum
    # (or that ran for a second or more) is held against the sustained one.
    capped = bool(clocks) and bool(clocks.get("sm_mhz")) and bool(clocks.get("sm_max_mhz")) and \
        clocks["sm_mhz"] < 0.9 * clocks["sm_max_mhz"]
    long_loop = total_ms > 1000.0 or capped
    peak = peaks["bf16_tflops_sustained"] if long_loop else peaks["bf16_tflops"]
    traffic = load_traffic(workload)
    peak_kind = "%s %s cuBLAS bf16 GEMM" % (peaks["source"], "sustained" if long_loop else "burst")
    if sparse:
        peak *= 2.0  # 2:4 sparse tensor-core peak = 2 x dense, dense-equivalent FLOPs
        peak_kind = "2 x " + peak_kind + " (2:4 sparse rate)"
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT, "frac": achieved / peak,
                "traffic": traffic, "peak_kind": peak_kind,
                "frac_of_nominal_2250": achieved / NOMINAL_DENSE_TFLOPS * (0.5 if sparse else 1.0),
                "launch_ms_avg": avg_launch_ms,
                "launch_ms_serialised_median": float(np.median(per_launch))}
    if resolved == 106 and not sparse:
        # Decode-shaped GEMM: HBM-bound; report bytes against measured HBM copy bandwidth.
        nbytes = 2.0 * (M * K + N * K + M * N)
        gbs = nbytes / (avg_launch_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": gbs / peaks["hbm_gbs"], "traffic": traffic, "algorithmic_bytes": nbytes,
                    "peak_kind": "%s HBM copy" % peaks["source"], "tflops": achieved,
                    "launch_ms_avg": avg_launch_ms,
                    "launch_ms_serialised_median": float(np.median(per_launch))}
    if probe_clk:
        sms = kb_sm_count(torch, local)
        clk_peak = sms * DENSE_FLOP_PER_CLK_SM * (2.0 if sparse else 1.0) * probe_clk["sm_mhz"] * 1e6 / 1e12
        roofline.update({"effective_sm_mhz": probe_clk["sm_mhz"], "frac_of_clock_peak": achieved / clk_peak,
                         "clock_peak_tflops": clk_peak, "clock_probe": probe_clk})
    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic",
        "config": {"workload": workload, "M_per_rank": M, "M_global": M_global, "N": N, "K": K, "layout": "RC",
                   "version": version, "rung": resolved,
                   "rung_name": kb.version_name(resolved) if isinstance(resolved, int) else resolved,
                   "accumulate": "fp32", "inputs": "N(0,1)/sqrt(K), torch generator per rank",
                   "l2": "3 rotating input sets (%.0f MiB A+B per rank) > 126 MB L2" %
                         (NSETS * (M * K + N * K) * 2 / 2**20),
                   "parallelism": "M-sharded x%d, B broadcast once (NCCL)" % world if world > 1 else "1 GPU"},
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": M * N * 2, "steps": args.e2e_steps, "finite": ok_e2e,
                "pipelining": "copy-in / GEMM / copy-out on three streams, two buffer sets"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "broadcast_ms": bcast_ms,
        "broadcast_gemm": bcast_gemm,
        "cublas": cublas,
        "parity": parity,
    }
    if extras:
        out.update(extras)
    if sparse:
        out["metric"] = "2:4 sparse FP16 RC GEMM TFLOP/s (dense-equivalent 2MNK) @ M=N=K=8192"
        out["useful_tflops"] = value / 2.0
        out["packer"] = packer
    if world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline_port(M, N, K, args.cpu_seconds)
            cb = out["cpu_baseline"]
            cb["cpu_model"] = cpu_model()
            cb["extrapolated_s_full_workload"] = 2.0 * M * N * K / (cb["value"] * 1e12)
            try:
                cb["reference_1core"] = cpu_reference_1core(M, N, K)
            except Exception as e:
                cb["reference_1core"] = {"unavailable": str(e)}
        except Exception as e:
            out["cpu_baseline"] = {"unavailable": str(e)}
    print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
