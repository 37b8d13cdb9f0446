"""Throughput of the CKKS key-switching hot path on B200: BASELINE config 2 (the headline microbenchmark).

A step is one pass of the hot path over one batch of 64 ciphertexts at N = 2^16 (24 x 50-bit Q limbs + 8 x 50-bit
special primes, dnum 3) whose residues are uniform random mod each prime (seeded): a forward + inverse NTT pass over
the batch (3072 rows each way) and the batch's key switches, 1 relinearization and the 16 rotations by 2^k,
k = 0..15. Rotation by 2^15 is the identity at N = 2^16 (g = 5^0 = 1) and runs as a copy, so 16 key switches per
ciphertext are counted (1024 per step per GPU). The 16 rotations of a ciphertext share one ModUp (hoisting, the
reference's Rotator::Hoisted); each still runs its own key inner product and ModDown. `plain_rotation_ks_per_s`
reports unhoisted rotations of the same batch. `value` = key switches per second over the whole job with the inputs
resident in HBM; `e2e` = the same step through the public API with the inputs copied in from pinned host memory and
the step's result (the summed outputs) copied back, inside the timed region.

Multi-GPU: one process per GPU, every rank its own batch (independent ciphertexts, keys replicated; no collective on
the data path): weak scaling, time = max over ranks.

--impl reference: the reference's CPU path for the same workload (the oracle port of crates/pc-host, all host
threads), rank 0 only; the same metric.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "key-switches/s at N=2^16 (config 2: 24+8 x 50-bit limbs, dnum 3, batch 64)"
UNIT = "key-switches/s"
BATCH = 64
ROT_STEPS = [1 << k for k in range(16)]  # 2^15 is the identity at N = 2^16
KS_PER_CT = 1 + sum(1 for s in ROT_STEPS if s % (1 << 15))


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=BATCH, help="ciphertexts per GPU (profiling cases only)")
    ap.add_argument("--profile", action="store_true",
                    help="the timed steps only (no e2e, plain-rotation, attention or CPU legs): the ncu case")
    ap.add_argument("--part", choices=["all", "projection", "attention", "block", "bootstrap", "model"],
                    default="all",
                    help="projection / attention: only that timing (one GPU; the timed steps in the NVTX range "
                         "'projection_step' / 'attention_step', the ncu case)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi samples during the timed region: median SM MHz under load and the throttle reasons seen."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ CPU path
_CPU = {}


def cpu_model():
    """The host CPU's model name (/proc/cpuinfo), for the baseline's record."""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_step(o, x):
    """The GPU step's work for one ciphertext on the oracle port (crates/pc-host restated): the NTT + INTT pass over its
    Q rows, the relinearized product, the 16 rotations 2^0..2^15 hoisted (one ModUp; each its own inner product and
    ModDown; 2^15 is the identity, a copy), the sum of the 17 outputs: KS_PER_CT key switches."""
    import numpy as np

    from tests import _oracle as O

    top = o.nq - 1
    rows = np.ascontiguousarray(x[:, : o.nq]).reshape(-1, o.n).copy()
    O.lib().orc_ntt_batch(o.h, rows, rows.shape[0], 0)
    O.lib().orc_ntt_batch(o.h, rows, rows.shape[0], 1)
    acc = o.mult(x, x, top)
    for r in o.rotate_hoisted(x, ROT_STEPS, top):
        acc = o.add(acc, r, top)
    return acc


def cpu_rate(samples, threads=None):
    """Key switches per second of the oracle port on this host's cores: `samples` GPU-shaped steps of one config-2
    ciphertext (_cpu_step, KS_PER_CT key switches each) on `threads` threads (default: every host thread). Returns
    (rate, threads, seconds)."""
    import numpy as np

    from perseus_b200 import fhe
    from tests import _oracle as O

    if not _CPU:
        # every host thread, whatever OMP_NUM_THREADS a launcher set (torchrun sets 1 per process)
        O.lib().orc_set_threads(len(os.sched_getaffinity(0)))
        ch = fhe.config2_chain()
        o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
        gal = [1] + [fhe.rotation_galois(st, ch.log_n) for st in ROT_STEPS if st % (ch.n // 2)]
        o.keygen(0, 192, 3.2, gal)
        rng = np.random.default_rng(0)
        x = o.ct()
        for r in range(o.nq):
            x[:, r] = rng.integers(0, ch.q[r], (2, o.n), dtype=np.uint64)
        _CPU.update(o=o, x=x)
    o, x = _CPU["o"], _CPU["x"]
    O.lib().orc_set_threads(threads or len(os.sched_getaffinity(0)))
    cores = O.lib().orc_get_threads()
    t0 = time.perf_counter()
    for _ in range(samples):
        _cpu_step(o, x)
    dt = time.perf_counter() - t0
    return samples * KS_PER_CT / dt, cores, dt


def run_reference(a):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    for _ in range(max(a.warmup, 1)):
        cpu_rate(1)
    times, cores = [], 0
    for _ in range(a.steps):
        _, cores, dt = cpu_rate(1)
        times.append(dt)
    rate = len(times) * KS_PER_CT / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic (uniform residues, seeded)",
        "config": {"workload": "config 2, one ciphertext per step: NTT + INTT pass over its 48 Q rows, 1 relin + 16 "
                               "hoisted rotations 2^0..2^15 (2^15 = identity copy; 16 key switches counted), the 17 "
                               "outputs summed: the GPU step's work per ciphertext",
                   "limbs": "24+8 x 50-bit", "dnum": 3},
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "one GPU-shaped step of one config-2 ciphertext per timed step (oracle port of "
                                   "crates/pc-host, OpenMP over rows)"},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ GPU path
def fp64_rate(L):
    """FP64 FMAs per second (T/s) of this GPU: the library's dependent-chain FMA loop on 4 blocks per SM, one warm-up
    launch, then one launch of about 30 ms timed with CUDA events on the launching stream. Returns (T/s, ms)."""
    import ctypes as C

    import torch

    sink = torch.empty(4096, dtype=torch.float64, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    n = L.lib().pcb_fp64_fma_loop(C.c_void_p(sink.data_ptr()), 20000, stream)
    if n < 0:
        raise RuntimeError(f"pcb_fp64_fma_loop: {n}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    n = L.lib().pcb_fp64_fma_loop(C.c_void_p(sink.data_ptr()), 400000, stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    return n / (ms * 1e-3) / 1e12, ms


def run_ours(a):
    import torch

    from perseus_b200 import _lib as L
    from perseus_b200 import fhe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    BATCH = a.batch
    ch = fhe.config2_chain()
    s = fhe.Session(ch, rot_steps=ROT_STEPS, k_max=BATCH, seed=0)
    n, nq, rows = ch.n, len(ch.q), ch.rows
    # the batch: residues uniform mod each prime, seeded per rank
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    x = torch.zeros((BATCH, 2, rows, n), dtype=torch.int64, device="cuda")
    for r in range(nq):
        x[:, :, r].random_(0, ch.q[r], generator=g)
    ct = fhe.Ct(x, nq - 1, 2.0**40, n // 2)
    ntt_rows = BATCH * 2 * nq
    nbuf = torch.empty((ntt_rows, n), dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def step(inp, ntt_t=None):
        # NTT / INTT pass over the batch's Q rows (3072 rows each way)
        nbuf.view(BATCH, 2, nq, n).copy_(inp.data[:, :, :nq])
        if ntt_t is not None:
            ntt_t[0].record(stream)
        s.ntt_batch(nbuf, ntt_rows, inverse=False)
        if ntt_t is not None:
            ntt_t[1].record(stream)
        s.ntt_batch(nbuf, ntt_rows, inverse=True)
        # 1 relinearization + 16 rotations (2^15: the identity copy), each output materialized, then summed into
        # one result in one pass
        outs = [s.mult(inp, inp)]
        outs += s.rotate_hoisted(inp, ROT_STEPS)  # one ModUp shared by the 16 steps (the reference's Hoisted)
        return s.sum(outs, out=outs[0])

    for _ in range(a.warmup):
        step(ct)
    torch.cuda.synchronize()
    # device-resident timing: 1.5 GiB of residues per batch, larger than the 126 MB L2 (no flush needed)
    clocks = Clocks(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    l0 = L.lib().pcb_launch_count()
    t0, t1 = ev(), ev()
    ntt_ev = [(ev(), ev()) for _ in range(a.steps)]
    t0.record(stream)
    for i in range(a.steps):
        step(ct, ntt_ev[i])
    t1.record(stream)
    torch.cuda.synchronize()
    launches = L.lib().pcb_launch_count() - l0
    barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / a.steps
    ntt_ms = sum(b.elapsed_time(e) for b, e in ntt_ev) / a.steps
    if a.profile:
        if rank == 0:
            print(json.dumps({"profile": True, "batch": BATCH, "ms_per_step": ms, "ntt_fwd_ms": ntt_ms,
                              "gpu_launches": int(launches)}), flush=True)
        return
    # e2e through the public API: every step copies its batch in from pinned host memory and its summed result out.
    # Double-buffered: the next batch's host->device copy and the previous result's device->host copy run on their
    # own streams while the step computes; the timed region ends when the last result is on the host.
    host_in = torch.empty((BATCH, 2, nq, n), dtype=torch.int64, pin_memory=True)
    host_in.copy_(x[:, :, :nq])
    host_out = [torch.empty((BATCH, 2, nq, n), dtype=torch.int64, pin_memory=True) for _ in range(2)]
    bufs = [fhe.Ct(torch.zeros_like(x), nq - 1, 2.0**40, n // 2) for _ in range(2)]
    cin, cout = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]

    # per (ciphertext, part) slice: rows 0..nq of a part are contiguous on both sides, so each is one direct
    # host<->device copy (a copy through the strided view of all parts would stage 1.6 GB in a device temporary)
    def fetch(b):
        with torch.cuda.stream(cin):
            for c in range(BATCH):
                for part in range(2):
                    bufs[b].data[c, part, :nq].copy_(host_in[c, part], non_blocking=True)
            in_ready[b].record(cin)

    barrier()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record(stream)
    cin.wait_event(e0)
    fetch(0)
    for i in range(a.steps):
        b = i % 2
        if i + 1 < a.steps:
            if i >= 1:
                cin.wait_event(in_free[1 - b])  # step i - 1 has finished reading that buffer
            fetch(1 - b)
        stream.wait_event(in_ready[b])
        res = step(bufs[b])
        in_free[b].record(stream)
        done = torch.cuda.Event()
        done.record(stream)
        cout.wait_event(done)
        with torch.cuda.stream(cout):
            for c in range(BATCH):
                for part in range(2):
                    host_out[b][c, part].copy_(res.data[c, part, :nq], non_blocking=True)
        res.data.record_stream(cout)
    stream.wait_stream(cout)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / a.steps
    barrier()
    # max over ranks
    t = torch.tensor([ms, e2e_ms, ntt_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, ntt_ms = t.tolist()
    ks = world * BATCH * KS_PER_CT
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm = peaks.get("hbm_gbs") or 6650.0
    ntt_bytes = 2 * ntt_rows * n * 8
    ntt_gbs = ntt_bytes / (ntt_ms * 1e-3) / 1e9
    # the same pass against the FP64 pipe, which is what bounds it: per N = 2^16 row, 16 stages x 2^15 butterflies of 8
    # FP64 operations (six for the exact product, the sum and the difference), the round reductions (3 per word, two
    # rounds), the column pass's twist product (6 per word), the conversion in (1) and the canonical form out (9)
    fp64_ops_row = 16 * (n // 2) * 8 + 2 * 3 * n + 6 * n + n + 9 * n
    fp64_tops = fp64_ops_row * ntt_rows / (ntt_ms * 1e-3) / 1e12
    fp64_nominal = 64 * 148 * 1.965e9 / 1e12  # FP64 FMA per clock per SM x SMs x max clock
    fp64_peak, fp64_peak_ms = fp64_rate(L)
    traffic = None
    try:
        traffic = json.load(open(os.path.join(ROOT, "profiles", "ntt_fwd_traffic.json")))["bytes_per_3072_row_pass"]
    except Exception:
        pass
    # The key switches of the step against both rooflines, over the whole timed step (it also holds the NTT pass and
    # the output sum: a lower bound on the key switches' own rates). Bytes: the algorithmic HBM traffic of one hybrid
    # key switch of one polynomial (c1 and c0 read, both output parts written: 4 L rows) plus the key (2 dnum (L + K)
    # rows, read once per batch); FP64 operations: every NTT row of the step (ModUp: L INTT + dnum (L + K) - L NTT
    # rows per ModUp; ModDown: 2 K INTT + 2 L NTT rows), the conversions' exact products (6 operations each: ModUp
    # dnum x alpha sources x (L + K - alpha) targets, ModDown 2 x K x L per coefficient) and the inner products'
    # (2 dnum (L + K) per coefficient, 7 operations with the sum). The relinearization has its own ModUp; the 15
    # rotations share one (hoisted) and each has its own ModDown and inner product.
    L_, K_, D_ = nq, rows - nq, ch.dnum
    alpha = -(-L_ // D_)
    R_ = n * 8
    real_rot = sum(1 for st in ROT_STEPS if st % (n // 2))
    ks_step = BATCH * (1 + real_rot)
    ks_bytes = BATCH * (1 + real_rot) * 4 * L_ * R_ + (1 + real_rot) * 2 * D_ * (L_ + K_) * R_
    modup_rows, moddown_rows = L_ + (D_ * (L_ + K_) - L_), 2 * K_ + 2 * L_
    ntt_rows_step = BATCH * (2 * modup_rows + (1 + real_rot) * moddown_rows)
    conv_macs = BATCH * n * (2 * D_ * alpha * (L_ + K_ - alpha) + (1 + real_rot) * 2 * K_ * L_)
    kip = BATCH * n * (1 + real_rot) * 2 * D_ * (L_ + K_)
    ks_fp64 = ntt_rows_step * fp64_ops_row + 6 * conv_macs + 7 * kip
    ks_gbs = ks_bytes / (ms * 1e-3) / 1e9
    ks_tops = ks_fp64 / (ms * 1e-3) / 1e12
    # plain (unhoisted) rotations of the same batch, for comparison: one key switch per rotation, ModUp included
    r0, r1 = ev(), ev()
    s.rotate(ct, 1)
    r0.record(stream)
    for _ in range(2):
        s.rotate(ct, 1)
    r1.record(stream)
    torch.cuda.synchronize()
    plain_ks = world * BATCH / (r0.elapsed_time(r1) / 2 * 1e-3)
    h2d, d2h = host_in.numel() * 8, host_out[0].numel() * 8
    del s, x, nbuf, bufs, host_in, host_out, ct, res
    torch.cuda.empty_cache()
    attn, attn_err = attention_decode(a, world, rank, barrier, dist)
    proj = projection(a, world, barrier, dist)
    blk = block_decode(a, world, barrier, dist)
    blk["batch_of_4"] = block_decode(a, world, barrier, dist, seqs=4)
    bts = bootstrap(a, world, barrier, dist)
    mdl = model_decode(a, world, barrier, dist)
    if rank == 0:
        line = {
            "metric": METRIC, "value": ks / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64", "data": "synthetic (uniform residues mod each prime, seeded)",
            "config": {"workload": "config 2: per GPU 64 ciphertexts, NTT+INTT pass (3072 rows) + 1 relin + 16 "
                                   "rotations 2^0..2^15 (2^15 = identity copy, 16 key switches / ct counted)",
                       "N": n, "limbs": "24+8 x 50-bit", "dnum": 3, "batch_per_gpu": BATCH,
                       "parallelism": f"replicas x{world} (independent ciphertexts, no collective)",
                       "l2": "inputs larger than L2 (1.5 GiB of residues per batch)"},
            "e2e": {"value": ks / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "roofline": {"kernel": "ntt fwd (fwd_cols + fwd_rows) over the batch's 3072 rows", "bound": "hbm",
                         "achieved": ntt_gbs, "peak": hbm, "unit": "GB/s", "frac": ntt_gbs / hbm,
                         "traffic": traffic, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                         "ms": ntt_ms, "algorithmic_bytes": ntt_bytes,
                         "fp64_pipe": {"ops_per_row": fp64_ops_row, "achieved_tops": fp64_tops, "peak_tops": fp64_peak,
                                       "frac": fp64_tops / fp64_peak,
                                       "peak_source": f"measured: FP64 FMA loop (pcb_fp64_fma_loop, {fp64_peak_ms:.0f} ms, "
                                                      "CUDA events)", "nominal_tops": fp64_nominal}},
            "keyswitch_roofline": {
                "kernels": "the step's key switches (ModUp, inner products, ModDown) over the whole step time",
                "key_switches_per_step": ks_step,
                "hbm": {"algorithmic_bytes": ks_bytes, "achieved": ks_gbs, "peak": hbm, "unit": "GB/s",
                        "frac": ks_gbs / hbm},
                "fp64_pipe": {"ops": ks_fp64, "achieved_tops": ks_tops, "peak_tops": fp64_peak,
                              "frac": ks_tops / fp64_peak, "floor_ms": ks_fp64 / (fp64_peak * 1e12) * 1e3},
                "bound": "fp64"},
            "clocks": clk,
            "attn_decode_ms_per_token": attn,
            "attn_decode_max_abs_err_vs_fp64": attn_err,
            "plain_rotation_ks_per_s": plain_ks,
            "projection": proj,
            "attention_block": blk,
            "bootstrap": bts,
            "model_decode": mdl,
        }
        if world == 1 and not a.no_cpu_baseline:
            try:
                rate, _, _ = cpu_rate(1)  # the estimate that sizes a ~10 s sample
                ns = max(2, min(200, int(10.0 * rate / KS_PER_CT)))
                rate, cores, dt = cpu_rate(ns)
                line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                                        "sample": f"{ns} GPU-shaped steps of one config-2 ciphertext ({ns * KS_PER_CT} "
                                                  f"key switches: relin + 16 hoisted rotations + NTT pass + sum; "
                                                  f"{dt:.1f} s)", "cpu_model": cpu_model()}
                # pc-host's default pool caps its threads at 36 (crates/pc-hostrt/src/lib.rs:219-226)
                capped = min(cores, 36)
                if capped != cores:
                    r36, _, _ = cpu_rate(max(1, ns * capped // cores), capped)
                    line["cpu_baseline"]["value_min_cores_36"] = r36
                else:
                    line["cpu_baseline"]["value_min_cores_36"] = rate
                line["cpu_baseline"]["threads_note"] = f"all {cores} host threads; min(cores, 36) = {capped}"
            except Exception as e:  # the baseline is reported, never required
                line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": None, "kind": "port",
                                        "sample": f"failed: {e}"}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def attention_decode(a, world, rank, barrier, dist):
    """Encrypted attention decode ms/token (the step with the KV cache resident in HBM, CUDA events, max over ranks):
    config 1 (one head, N = 2^14, 32 tokens) on rank 0's GPU, and config 3's attention core (12 heads x 64, 128
    tokens, N = 2^16 with the 24-limb chain), heads sharded over the ranks (perseus_b200.shard.head_range, no
    communication: the per-head outputs stay on their GPU)."""
    import numpy as np
    import torch

    from perseus_b200 import attention as A
    from perseus_b200 import fhe, shard

    out, err = {}, {}
    for name, ch, tokens, heads in (("config1_1head_N2^14_32tok", fhe.config1_chain(), 32, 1),
                                    ("config3_12heads_N2^16_128tok", fhe.config2_chain(), 128, 12)):
        # config 1 runs on every rank (rank 0 reports it) on BASELINE's data (default_rng(0): K, V then Q); config
        # 3's heads are split, at most one apart, each rank drawing its own
        rng = np.random.default_rng(0 if heads == 1 else 100 + rank)
        mine = heads if heads == 1 else len(shard.head_range(heads, world, rank))
        lay = A.Layout(64, tokens, ch.n // 2, radix_bits=3)  # radix-3 ladders (rotate_sum groups)
        s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=mine, seed=0)
        top = len(ch.q) - 1
        caches, qs, plain = [], [], []
        for _ in range(mine):
            c = A.KVCache(s, lay, top)
            K, V = rng.normal(0, 1, (tokens, 64)) / 8, rng.normal(0, 1, (tokens, 64)) / 8
            qv = rng.normal(0, 1, 64) / 8
            c.load(K, V)
            caches.append(c)
            qs.append(A.encrypt_query(s, qv, lay, top, ch.q[top]))
            plain.append((qv, K, V))
        cache = caches[0] if mine == 1 else A.HeadBatch(s, caches)
        q = qs[0] if mine == 1 else s.stack(qs)
        coeffs = A.softmax_poly(tokens)
        # eager steps (host dispatch of every op), then the same step replayed as one CUDA graph
        graph = A.DecodeGraph(s, cache, coeffs, ch.q, q)
        times = []
        for run in (lambda: A.attend(s, q, cache, coeffs, ch.q), lambda: graph(q)):
            for _ in range(max(a.warmup, 3)):
                run()
            torch.cuda.synchronize()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push("attention_step")
            e0.record()
            for _ in range(a.steps):
                run()
            e1.record()
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / a.steps)
        t = torch.tensor(times, dtype=torch.float64, device="cuda")
        if dist and heads > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[name] = t[1].item()
        out[name + "_eager"] = t[0].item()
        # decrypted output of this rank's first head against fp64 attention with the same polynomial softmax
        res = graph(q)
        qv, K, V = plain[0]
        got = s.decrypt_slots(res, 0).real[:64]
        err[name] = float(np.abs(got - A.plain_attention(qv, K, V, coeffs)).max())
        del s, caches, qs, cache, q, graph, res
        torch.cuda.empty_cache()
    return out, err


def projection(a, world, barrier, dist):
    """GPT-2's attention projections at config 3's ring (N = 2^16, 24+8 limbs): the Q, K and V linears of one
    activation (768 of the padded 1024, weights N(0, 0.02), shared prepared input and babies) and the output linear,
    ms per token with CUDA events (every rank runs the same replica; max over ranks), and the decrypted error against
    fp64 x W + b."""
    import numpy as np
    import torch

    from perseus_b200 import fhe
    from perseus_b200 import linear as LIN

    ch = fhe.config2_chain()
    geo = LIN.geometry(ch.n // 2, 1024)
    radix = 3
    s = fhe.Session(ch, rot_steps=geo.rot_steps(radix), k_max=3, seed=0)  # Q, K, V run as one batch of 3
    rng = np.random.default_rng(7)
    n, top = 768, len(ch.q) - 1
    x = rng.normal(0, 1, n)
    Ws = [rng.normal(0, 0.02, (n, n)) for _ in range(4)]
    bs = [rng.normal(0, 0.02, n) for _ in range(4)]
    xc = s.encrypt(LIN.input_vector(x, geo), top=top, scale=2.0**40, slots=geo.slots)
    qkv = [LIN.encode(s, W, geo, top, xc.scale, bias=b) for W, b in zip(Ws[:3], bs[:3])]
    out = LIN.encode(s, Ws[3], geo, top, xc.scale, bias=bs[3])
    times = []
    for run in (lambda: LIN.linear_multi(s, xc, qkv, radix), lambda: LIN.linear(s, xc, out, radix)):
        for _ in range(max(a.warmup, 3)):
            run()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("projection_step")
        e0.record()
        for _ in range(a.steps):
            run()
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / a.steps)
    t = torch.tensor(times, dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ys = LIN.linear_multi(s, xc, qkv, radix)
    err = max(float(np.abs(LIN.output_values(s.decrypt_slots(y).real, geo, n) - (x @ W + b)).max())
              for y, W, b in zip(ys, Ws, bs))
    del s, qkv, out, xc, ys
    torch.cuda.empty_cache()
    form = "double-hoisted: babies in the extended basis" if geo.ext else "hoisted babies"
    return {"workload": "GPT-2 attention projections, one token: Q/K/V linears (768 of 1024, shared input) and the "
                        f"output linear, N=2^16 24+8 limbs, {geo.npts} weight plaintexts each ({geo.bstep} baby x "
                        f"{geo.gstep} giant, {form}), radix-3 ladders",
            "qkv_ms": t[0].item(), "out_ms": t[1].item(), "max_abs_err_vs_fp64": err}


def block_decode(a, world, barrier, dist, seqs=1):
    """Config 3's attention block, one token per step: the polynomial LayerNorm (gamma, beta folded into Q/K/V), Q/K/V
    projections, the token's K and V pushed into the lane cache (128 tokens in 4 blocks of 32, all 12 heads per
    block), attention over the cache, output projection, residual (perseus_b200.block; N = 2^16 with the 24-limb
    chain, weights N(0, 0.02), biases, gamma 1 + N(0, 0.02), activation N(0, 1)).
    The cache starts with client-encrypted tokens and grows by one per step up to its 128; ms per token with CUDA
    events (max over ranks), and the last step's decrypted error against the fp64 step. On N GPUs a single sequence's
    4 cache blocks are split over the ranks (LaneCache shard=: each rank attends over its share, one all_gather of the
    partial outputs summed mod p on every rank; the LayerNorm and the projections run on every rank); with seqs > 1
    every rank decodes its own sequences (replicas, tokens/s over all GPUs)."""
    import numpy as np
    import torch

    from perseus_b200 import attention as A
    from perseus_b200 import block as B
    from perseus_b200 import fhe

    ch = fhe.config2_chain()
    lay = B.layout(ch.n // 2, 1024, heads=12, head_dim=64, tokens=128, radix_bits=3)
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=max(lay.blocks, 3) * seqs, seed=0)
    rng = np.random.default_rng(11)
    warm, steps = max(a.warmup, 3), min(a.steps, 64)  # the cache holds 128 tokens: the steps fill its last lanes
    n, pre, top = 768, lay.tokens - warm - steps, len(ch.q) - 1
    w = B.Weights(*[rng.normal(0, 0.02, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])
    gamma, beta = 1 + rng.normal(0, 0.02, n), rng.normal(0, 0.02, n)
    wf, norm = B.fold_norm(w, gamma, beta), B.NormCfg()
    Ks = [rng.normal(0, 1, (pre, n)) / 8 for _ in range(seqs)]
    Vs = [rng.normal(0, 1, (pre, n)) / 8 for _ in range(seqs)]
    # one sequence: its cache blocks split over the ranks (latency); several: every rank decodes its own (throughput)
    shard_ = (world, int(os.environ.get("RANK", "0"))) if world > 1 and seqs == 1 else None
    cache = B.LaneCache(s, lay, top - 10, seqs=seqs, shard=shard_)
    cache.load(Ks if seqs > 1 else Ks[0], Vs if seqs > 1 else Vs[0])
    coeffs = A.softmax_poly(lay.tokens)
    xs = [[rng.normal(0, 1, n) for _ in range(seqs)] for _ in range(warm + steps)]
    cts = [s.stack([s.encrypt(B.LIN.input_vector(x, lay.geo), top=top, scale=2.0**40, slots=lay.slots) for x in xq])
           for xq in xs]
    Kp, Vp = [Ks[0]], [Vs[0]]
    y = None
    for i in range(warm):
        y = B.decode(s, cts[i], wf, cache, coeffs, ch.q, norm=norm, residual=True)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("block_step")
    e0.record()
    for i in range(warm, len(cts)):
        y = B.decode(s, cts[i], wf, cache, coeffs, ch.q, norm=norm, residual=True)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device="cuda")  # per step of all sequences
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    # sequence 0's fp64 step of the last token, with its earlier tokens' K and V rows appended as the cache saw them
    for xq in xs[:-1]:
        xn = norm.plain(xq[0]) * gamma + beta
        Kp.append((xn @ w.wk + w.bk)[None])
        Vp.append((xn @ w.wv + w.bv)[None])
    want = B.plain_decode(norm.plain(xs[-1][0]) * gamma + beta, w, np.vstack(Kp), np.vstack(Vp), coeffs, 12, 64) + \
        xs[-1][0]
    got = B.LIN.output_values(s.decrypt_slots(y, 0).real, lay.geo, n)
    err = float(np.abs(got - want).max())
    del s, cache, cts, y
    torch.cuda.empty_cache()
    out = {"workload": "config 3 attention block, one token: LayerNorm (degree-7 inverse square root), Q/K/V "
                       "projections (768 of 1024), push into a 128-token lane cache (4 blocks x 32 tokens, 12 heads "
                       "x 64 per block), attention with the degree-7 polynomial softmax, output projection, "
                       "residual; N=2^16 24+8 limbs, radix-3 ladders, eager",
           "ms_per_token": t.item(), "timed_tokens": steps, "max_abs_err_vs_fp64": err,
           "tokens_in_cache_at_end": pre + len(xs),
           "sharding": f"cache blocks over {world} GPU(s): {lay.blocks} blocks, one all_gather of the partial "
                       "outputs per token" if world > 1 else "one GPU"}
    if seqs > 1:
        out = {"sequences_per_gpu": seqs, "ms_per_step": t.item(), "tokens_per_s_all_gpus": world * seqs / (t.item() * 1e-3),
               "parallelism": f"replicas x{world} (independent sequences)",
               "max_abs_err_vs_fp64_seq0": err}
    return out


def bootstrap(a, world, barrier, dist):
    """Config 4: CKKS bootstrapping at N = 2^16 with full slots (2^15), a level-0 ciphertext of uniform [-1, 1] slot
    values (seeded) refreshed to 12 usable levels (perseus_b200.bootstrap: ModRaise, CoeffToSlot in 3 BSGS groups,
    conjugate split, EvalMod by the degree-63 Chebyshev interpolant with 3 double angles, SlotToCoeff in 3 groups) on
    the 29 + 11 limb chain (dnum 3, secret of Hamming weight 192). ms per bootstrap with CUDA events (every rank runs a
    replica; max over ranks) and the refreshed ciphertext's decrypted error against the input slots."""
    import numpy as np
    import torch

    from perseus_b200 import bootstrap as BS
    from perseus_b200 import fhe

    ch = fhe.config4_chain()
    prm = BS.Params(ch.n, K=24, r=3, per_group=5)
    s = fhe.Session(ch, rot_steps=BS.rot_steps(prm), k_max=2, seed=0, h=192, sigma=3.2,
                    galois_extra=(BS.conj_galois(ch.n),))
    z = np.random.default_rng(12).uniform(-1, 1, prm.slots)
    ct = s.encrypt(z, top=0, scale=2.0**40, slots=prm.slots)
    bt = BS.Bootstrapper(s, prm, ch.q, ch.q[0])
    top = len(ch.q) - 1
    out = None
    for _ in range(max(a.warmup, 3)):
        out = bt(ct, top)
    steps = max(1, min(a.steps, 10))
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("bootstrap_step")
    e0.record()
    for _ in range(steps):
        out = bt(ct, top)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    got = s.decrypt_slots(out)
    err = got - z
    res = {"workload": "config 4: CKKS bootstrap, N=2^16, full slots (2^15), level 0 -> 12 usable levels, 29+11 x "
                       "50-bit limbs, dnum 3, h=192, EvalMod K'=24 degree 63 + 3 double angles, CoeffToSlot / "
                       "SlotToCoeff 3 groups of 5 FFT stages each",
           "ms_per_bootstrap": t.item(), "bootstraps_per_s_all_gpus": world * 1e3 / t.item(), "timed": steps,
           "levels_out": out.top, "max_abs_err": float(np.abs(err.real).max()),
           "rms_err": float(np.sqrt((err.real ** 2).mean())), "max_abs_imag": float(np.abs(got.imag).max()),
           "rotation_keys": len(BS.rot_steps(prm)) + 1}
    del s, ct, out, bt
    torch.cuda.empty_cache()
    return res


def model_decode(a, world, barrier, dist):
    """Config 5: GPT-2 small's 12 layers decoded on encrypted activations (perseus_b200.model: LayerNorm, attention
    over a 256-token encrypted cache per layer resident in HBM, MLP with the polynomial GELU, residuals, 4 refreshes
    per layer), N = 2^16 on config 4's chain, random-init weights N(0, 0.02); the caches start with client-encrypted
    tokens and grow by one per token. One warm-up token (it also encodes every plaintext once), then `steps` tokens
    (at most 4) timed with CUDA events (max over ranks), the last decrypted against the fp64 decode; on N GPUs every
    layer's 8 cache blocks are split over the ranks (one all_gather of the partial attention outputs per layer). Then
    4 sequences decoding together (one token each per step, every op on their batch): one warm-up step and `steps` (at
    most 2) timed; on N GPUs every rank decodes its own 4 sequences (replicas, no collective: tokens/s over all GPUs)."""
    import numpy as np
    import torch

    from perseus_b200 import bootstrap as BS
    from perseus_b200 import fhe
    from perseus_b200 import linear as LIN
    from perseus_b200 import model as M

    cfg = M.ModelCfg()
    ch = fhe.config4_chain()
    prm = BS.Params(ch.n, K=24, r=3, per_group=5)
    lay = M.B.layout(ch.n // 2, cfg.width, cfg.heads, cfg.head_dim, cfg.tokens, cfg.radix_bits)
    steps_rot = sorted(set(BS.rot_steps(prm)) | set(lay.rot_steps()))
    S4 = 4
    s = fhe.Session(ch, rot_steps=steps_rot, k_max=lay.blocks * S4, seed=0, h=192, sigma=3.2,
                    galois_extra=(BS.conj_galois(ch.n),))
    rng = np.random.default_rng(13)
    weights = [M.random_layer(rng) for _ in range(cfg.layers)]
    bt = BS.Bootstrapper(s, prm, ch.q, ch.q[0])
    shard_ = (world, int(os.environ.get("RANK", "0"))) if world > 1 else None

    def run(seqs, warm, steps, plan, shard):
        pre = cfg.tokens - warm - steps
        Ks = [[rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(seqs)] for _ in range(cfg.layers)]
        Vs = [[rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(seqs)] for _ in range(cfg.layers)]
        dec = M.Decoder(s, cfg, weights, ch.q, bt, shard=shard, seqs=seqs, plan=plan)
        dec.load(Ks if seqs > 1 else [k[0] for k in Ks], Vs if seqs > 1 else [v[0] for v in Vs])
        plain = [[Ks[l][0].copy(), Vs[l][0].copy()] for l in range(cfg.layers)]  # sequence 0's fp64 caches
        xs = [[rng.normal(0, 1, cfg.d) for _ in range(seqs)] for _ in range(warm + steps)]
        cts = [s.stack([s.encrypt(LIN.input_vector(x, lay.geo), top=0, scale=2.0**40, slots=lay.slots) for x in xq])
               for xq in xs]
        y = None
        for i in range(warm):
            y = dec.decode(cts[i])
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("model_step")
        e0.record()
        for i in range(warm, warm + steps):
            y = dec.decode(cts[i])
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device="cuda")
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        want = None
        for xq in xs:
            want = M.plain_decode(xq[0], weights, plain, cfg, dec.coeffs)
        got = LIN.output_values(s.decrypt_slots(y, 0).real, lay.geo, cfg.d)
        return t.item(), float(np.abs(got - want).max()), float(np.abs(want).max()), dec.plan

    # one sequence: its cache blocks split over the ranks (latency); four sequences: every rank decodes its own four
    # (independent sequences, no collective: throughput)
    ms1, err1, mx1, plan = run(1, 1, max(1, min(a.steps, 4)), None, shard_)
    ms4, err4, _, _ = run(S4, 1, max(1, min(a.steps, 2)), plan, None)
    res = {"workload": "config 5: GPT-2 small, 12 layers (768 wide, 12 heads x 64, MLP 3072), one token per step, "
                       "a 256-token encrypted KV cache per layer in HBM (8 blocks x 32 tokens), N=2^16 on 29+11 x "
                       "50-bit limbs, 4 refreshes (bootstraps) per layer, degree-7 polynomial LayerNorm / softmax / "
                       "GELU, eager",
           "ms_per_token": ms1, "timed_tokens": max(1, min(a.steps, 4)), "refreshes_per_token": 4 * cfg.layers,
           "max_abs_err_vs_fp64": err1, "max_abs_value": mx1,
           "batch_of_4": {"sequences_per_gpu": S4, "ms_per_step": ms4, "tokens_per_s_all_gpus": world * S4 / (ms4 * 1e-3),
                          "max_abs_err_vs_fp64_seq0": err4, "parallelism": f"replicas x{world} (independent sequences)"},
           "sharding": f"every layer's cache blocks over {world} GPU(s)" if world > 1 else "one GPU"}
    del s, bt, plan
    torch.cuda.empty_cache()
    return res


def main():
    a = parse()
    if a.part == "model":  # under torchrun every layer's cache blocks are split over the ranks (rank 0 prints)
        import torch

        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))

        def barrier():
            if dist:
                dist.barrier()

        out = {"part": "model", "n_gpus": world, **model_decode(a, world, barrier, dist)}
        if rank == 0:
            print(json.dumps(out), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if a.part == "bootstrap":
        print(json.dumps({"part": "bootstrap", **bootstrap(a, 1, lambda: None, None)}), flush=True)
        return
    if a.part == "projection":
        print(json.dumps({"part": "projection", **projection(a, 1, lambda: None, None)}), flush=True)
        return
    if a.part == "block":  # under torchrun the cache blocks are split over the ranks (rank 0 prints)
        import torch

        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))

        def barrier():
            if dist:
                dist.barrier()

        out = {"part": "block", "n_gpus": world, **block_decode(a, world, barrier, dist),
               "batch_of_4": block_decode(a, world, barrier, dist, seqs=4)}
        if rank == 0:
            print(json.dumps(out), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if a.part == "attention":
        ms, err = attention_decode(a, 1, 0, lambda: None, None)
        print(json.dumps({"part": "attention", "ms_per_token": ms, "max_abs_err_vs_fp64": err}), flush=True)
        return
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
