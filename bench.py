"""ArcLLM-B200 benchmark: Q4_K/Q6_K dequant-matvec HBM throughput on B200.

Headline workload (N=1 and every N): the Q6_K LM-head matvec, 152064 x 3584
(447,068,160 weight bytes), fp32 x ~ N(0,1).  One step = one pass of the LM
head over one activation vector.  At N>1 the rows are sharded over the ranks
(152064/N contiguous rows each) and the fp32 logits are all-gathered by the
matvec kernel itself over NVLink peer stores (`--collective nccl`: matvec +
ncclAllGather), so every rank ends the step with the full logits (strong
scaling).

Timing: W untimed warm-up steps, then K steps between barrier +
cuda.synchronize on both sides, CUDA events on the launching stream, max
over ranks.  The weights (447 MB) are larger than the 126 MB L2, so
consecutive steps read them from HBM; the smaller extra configs rotate
enough weight copies to exceed 3x L2.

Printed (rank 0, one JSON line): the contract keys plus `roofline` (dominant
kernel = the matvec; achieved = algorithmic bytes / mean kernel time vs the
measured HBM copy bandwidth), `cpu_baseline` (the reference's own CPU
matmul_q6_cpu timed on this host), `e2e` (the C-ABI host-IO call every
step: pinned host x copied in, the matvec -- with the all-gather at N>1 --
storing all logits into pinned mapped host memory, stream sync), `clocks`,
and `extra` (configs 0, 1b, 2, 3, 4 at N=1; the sharded forms at N>1).

`--impl reference` times the reference's CPU implementation of the same
workload (oracle/_ref, compiled from the reference sources; the restated
oracle where that library is absent) on all host cores, and prints the
same line with "impl": "reference".
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K/Q6_K matvec HBM GB/s (% of B200 peak); decode tok/s, Qwen2.5-7B shape"
LM_ROWS, HIDDEN, FFN = 152064, 3584, 18944
Q4B, Q6B = 144, 210
L2_BYTES = 126 * 1024 * 1024


def q_bytes(fmt, rows, k):
    return rows * (k // 256) * (Q4B if fmt == "q4k" else Q6B)


def matvec_alg_bytes(fmt, rows, k):
    """weights + x (fp32) + y (fp32): the algorithmic bytes of one matvec"""
    return q_bytes(fmt, rows, k) + 4 * k + 4 * rows


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def committed_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/*.json)"""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    return json.load(open(p)).get(name)


# --------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            cmd = ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "50"]
            if self.gpu_id is not None:
                cmd += ["-i", str(self.gpu_id)]
            self.proc = subprocess.Popen(cmd, stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # nvidia-smi can take a while to start on a many-GPU box: wait (bounded) for its first sample,
        # so the samples bracket the timed region however short it is
        t0 = time.time()
        while self._lines() == 0 and self.proc.poll() is None and time.time() - t0 < 5.0:
            time.sleep(0.02)

    def _lines(self):
        try:
            with open(self.f.name) as g:
                return sum(1 for ln in g if ln.strip())
        except OSError:
            return 0

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        n0, t0 = self._lines(), time.time()  # one more sample after the timed region (bounded)
        while self._lines() <= n0 and self.proc.poll() is None and time.time() - t0 < 1.0:
            time.sleep(0.02)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [l.strip().split(",") for l in self.f.read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                power.append(float(r[3]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def gpu_smi_id(torch, local_rank):
    try:
        p = torch.cuda.get_device_properties(local_rank)
        return "%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[local_rank]
        return local_rank


# --------------------------------------------------------------- cpu baseline
def host_cpu_model():
    """The host CPU's model name (first /proc/cpuinfo entry), or None."""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_baseline(seconds=10.0):
    """The reference's own matmul_q6_cpu (oracle/_ref) on a bounded sample of
    the LM head, 1 thread (the reference's form); the restated oracle is used
    only where the reference library is absent."""
    import numpy as np

    import oracle as O
    rows = 8192
    w = O.fill_q6k(rows, HIDDEN, 0x1A4D)
    x = O.normal_f32(HIDDEN, 0x1A4E)
    y = np.empty(rows, np.float32)
    kind = "reference" if O.ref is not None else "port"
    done, t0 = 0, time.perf_counter()
    while True:
        if O.ref is not None:
            O.ref.ref_matmul_q6(w, HIDDEN, rows, 1, x, None, y)
        else:
            O.orc.orc_matmul_q6(w, HIDDEN, rows, 1, x, None, y, 1)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 400:
            break
    gbs = done * matvec_alg_bytes("q6k", rows, HIDDEN) / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind, "cpu_model": host_cpu_model(),
            "sample": "%d passes over an 8192-row slice (%.1f MB) of the 152064x3584 Q6_K LM head, "
                      "x fp32, 1 thread, %.1f s" % (done, q_bytes("q6k", rows, HIDDEN) / 1e6, el)}


def run_reference(args):
    """--impl reference: the reference's CPU path on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    import oracle as O
    cores = os.cpu_count() or 1
    rows = 19008  # 1/8 of the LM head per step (bounded sample)
    w = O.fill_q6k(rows, HIDDEN, 0x2B5E)
    x = O.normal_f32(HIDDEN, 0x2B5F)
    y = np.empty(rows, np.float32)
    kind = "reference" if O.ref is not None else "port"
    rb = q_bytes("q6k", 1, HIDDEN)
    bounds = [rows * t // cores for t in range(cores + 1)]

    def part(t):
        r0, r1 = bounds[t], bounds[t + 1]
        if r1 <= r0:
            return
        wv = w[r0 * rb:r1 * rb]
        yv = np.empty(r1 - r0, np.float32)
        if O.ref is not None:
            O.ref.ref_matmul_q6(wv, HIDDEN, r1 - r0, 1, x, None, yv)
        else:
            O.orc.orc_matmul_q6(wv, HIDDEN, r1 - r0, 1, x, None, yv, 1)
        y[r0:r1] = yv

    def step():
        ts = [threading.Thread(target=part, args=(t,)) for t in range(cores)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = args.steps * matvec_alg_bytes("q6k", rows, HIDDEN) / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config1: Q6_K LM-head matvec 152064x3584, fp32 x; reference CPU path on a "
                               "19008-row (1/8) sample per step", "parallelism": "%d host threads" % cores},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": kind,
                         "cpu_model": host_cpu_model(),
                         "sample": "19008 rows x 3584 (55.9 MB) of the LM head per step, rows split over "
                                   "%d threads, reference matmul_q6_cpu per row" % cores},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the extra configs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-IO leg")
    ap.add_argument("--fmt", default="q6k", choices=["q6k", "q4k"], help="profiling override of the workload")
    ap.add_argument("--rows", type=int, default=LM_ROWS, help="profiling override of the workload")
    ap.add_argument("--k", type=int, default=HIDDEN, help="profiling override of the workload")
    ap.add_argument("--only", choices=["decode", "prefill", "extra", "matvec", "gateup"],
                    help="profiling: run only the config-3 decode, the config-4 prefill GEMMs, all extra "
                         "configurations, one matvec shape (--fmt/--rows/--k) or the fused gate/up "
                         "(--rows/--k) over rotating weight copies, and print the result")
    ap.add_argument("--launch", default="graph", choices=["graph", "stream"],
                    help="N=1 headline: the K timed launches captured in one CUDA graph and replayed once "
                         "(default), or launched one by one with per-launch CUDA events")
    ap.add_argument("--collective", default="nvlink", choices=["nvlink", "nccl"],
                    help="N>1: logits all-gather fused into the matvec over NVLink peer stores (default) or the "
                         "matvec followed by ncclAllGather")
    ap.add_argument("--no-overlap", action="store_true",
                    help="graph mode without programmatic dependent launch between the timed launches")
    ap.add_argument("--decode-prompt", type=int, default=256)
    ap.add_argument("--decode-new", type=int, default=128)
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    if args.only:
        import torch

        import arcllm_b200 as A
        torch.cuda.set_device(0)
        if args.only == "decode":
            res = run_decode(A, torch, measured_peaks()[0], args.decode_prompt, args.decode_new)
        elif args.only in ("matvec", "gateup"):
            res = run_one_matvec(A, torch, measured_peaks()[0], args.fmt, args.rows, args.k, args.steps,
                                 args.warmup, dual=args.only == "gateup")
        else:
            res = run_extra(A, A.lib(), torch, torch.device("cuda", 0),
                            C.c_void_p(torch.cuda.current_stream().cuda_stream), measured_peaks()[0],
                            which="prefill" if args.only == "prefill" else "all")
        print(json.dumps(res), flush=True)
        return 0

    import numpy as np
    import torch

    import arcllm_b200 as A

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    L = A.lib()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- headline: LM head (rows sharded over ranks) ----
    fmt, ROWS, K = args.fmt, args.rows, args.k
    headline = (fmt, ROWS, K) == ("q6k", LM_ROWS, HIDDEN)
    TY = A.GGML_Q6_K if fmt == "q6k" else A.GGML_Q4_K
    rows_per = ROWS // world
    r0 = rank * rows_per
    rb = q_bytes(fmt, 1, K)
    w = torch.empty(rows_per * rb + 16, dtype=torch.uint8, device=dev)
    A.call("arcllm_cuda_fill_" + fmt, C.c_void_p(w.data_ptr()), r0 * (K // 256), rows_per * (K // 256),
           0x1A4D, sp)
    # x ~ N(0,1) generated with the library's fixture stream (same as the oracle's)
    x = torch.empty(K, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(x.data_ptr()), 0, K, 0x1A4E, C.c_float(0.0),
           C.c_float(1.0), sp)
    y = torch.empty(rows_per, dtype=torch.float32, device=dev)
    logits = torch.empty(rows_per * world, dtype=torch.float32, device=dev)
    wp, xp, yp = C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr())

    rg = None
    if dist is not None and args.collective == "nvlink":
        from arcllm_b200.rank_gather import RankGather

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        rg = RankGather(rows_per * world, world, rank, exchange)
        barrier()

    def step():
        if rg is not None:  # one kernel: rows + NVLink peer stores of epoch-tagged words
            rg.step(wp, rows_per, K, xp, r0, sp, TY)
            return
        st = L.arcllm_cuda_matvec(TY, wp, rows_per, K, xp, None, C.c_float(0.0), None, None, yp, sp)
        if st:
            A.check(st, "matvec")
        if dist is not None:
            dist.all_gather_into_tensor(logits, y)

    for _ in range(args.warmup):
        step()
    barrier()
    # N=1: the K timed launches as one CUDA graph (no host launch gaps between passes; every pass
    # still streams all weights from HBM).  The epochs of the N>1 all-gather change per launch, so
    # those run as stream launches.
    graph = rendezvous = None
    # graph mode: consecutive launches overlap (programmatic dependent launch: a launch streams its weights
    # while its predecessor drains, then waits for it before reading x or writing the logits)
    overlap = args.launch == "graph" and not args.no_overlap
    if overlap:
        A.check(L.arcllm_cuda_set_launch_overlap(1), "launch overlap")
    if args.launch == "graph" and dist is None:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            for _ in range(args.steps):
                A.check(L.arcllm_cuda_matvec(TY, wp, rows_per, K, xp, None, C.c_float(0.0), None, None, yp, cs),
                        "matvec")
        graph.replay()  # upload; an untimed pass like the warm-up steps
        torch.cuda.synchronize()
    elif args.launch == "graph" and rg is not None:
        # N>1 with the fused all-gather: every launch carries its own epoch, so the K timed launches are
        # captured with epochs e+K+1 .. e+2K after an untimed graph of epochs e+1 .. e+K, and each graph is
        # replayed exactly once (every rank captures the same sequence).  Host launch gaps, which the flag
        # handshake would otherwise turn into waits of the other ranks, stay out of the timed region.
        # Between the two sits a one-launch graph replayed untimed right before the timed one: it ends on
        # every rank within a flag round trip of the others, so the ranks start their timed launches
        # together instead of at the host skew of the barrier (which the first timed launch would absorb).
        graphs = []
        for n_launch in (args.steps, 1, args.steps):
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_, capture_error_mode="thread_local"):
                cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
                for _ in range(n_launch):
                    rg.step(wp, rows_per, K, xp, r0, cs, TY)
            graphs.append(g_)
        barrier()
        graphs[0].replay()
        torch.cuda.synchronize()
        rendezvous = graphs[1]
        graph = graphs[2]
        del graphs
        # the first launch of a graph also uploads it to the device: upload the rendezvous and the timed
        # graph now (driver cuGraphUpload: no kernel runs, no epoch is consumed), outside the timed region
        cu = C.CDLL("libcuda.so.1")
        cu.cuGraphUpload.argtypes = [C.c_void_p, C.c_void_p]
        for g_ in (rendezvous, graph):
            r_ = cu.cuGraphUpload(C.c_void_p(g_.raw_cuda_graph_exec()), sp)
            if r_ != 0:
                raise RuntimeError("cuGraphUpload failed: %d" % r_)
        torch.cuda.synchronize()
    if overlap:
        A.check(L.arcllm_cuda_set_launch_overlap(0), "launch overlap")
    clk = ClockSampler(gpu_smi_id(torch, local_rank))
    clk.start()
    time.sleep(0.1)
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(0 if graph is not None else args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if rendezvous is not None:
        rendezvous.replay()
        # 2 ms of device wall-clock time after the rendezvous, the same on every rank whatever its SM
        # clock: the host has the timed graph queued before any rank starts it
        A.check(L.arcllm_cuda_stream_delay_us(2000, sp), "stream_delay")
    t_start.record()
    if graph is not None:
        graph.replay()
    for i in range(0 if graph is not None else args.steps):
        ev[i][0].record()
        if rg is not None:
            rg.step(wp, rows_per, K, xp, r0, sp, TY)
        else:
            st = L.arcllm_cuda_matvec(TY, wp, rows_per, K, xp, None, C.c_float(0.0), None, None, yp, sp)
            if st:
                A.check(st, "matvec")
        ev[i][1].record()
        if dist is not None and rg is None:
            dist.all_gather_into_tensor(logits, y)
    t_end.record()
    barrier()
    clocks = clk.stop()
    total_ms = t_start.elapsed_time(t_end)
    # per-launch events in stream mode; in graph mode the mean over the back-to-back replay
    kern_ms = (sum(a.elapsed_time(b) for a, b in ev) if ev else total_ms) / args.steps
    del graph, rendezvous
    bits = C.c_uint32(0)
    A.check(L.arcllm_cuda_device_error(sp, C.byref(bits)), "device_error")
    if dist is not None:
        tt = torch.tensor([total_ms, kern_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, kern_ms = float(tt[0]), float(tt[1])
    ms_per_step = total_ms / args.steps
    alg_total = matvec_alg_bytes(fmt, rows_per * world, K)
    value = alg_total / (ms_per_step * 1e-3) / 1e9
    alg_shard = matvec_alg_bytes(fmt, rows_per, K)
    achieved = alg_shard / (kern_ms * 1e-3) / 1e9
    hbm_peak, _, peak_src = measured_peaks()
    traffic = committed_traffic("lmhead_q6k_%d" % world) if headline else None

    # ---- e2e through the C-ABI host-IO entry point (rank-local shard + all-gather) ----
    xh = torch.empty(K, dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    yh = torch.empty(rows_per, dtype=torch.float32).pin_memory()
    xd = torch.empty(K, dtype=torch.float32, device=dev)
    lh = torch.empty(rows_per * world, dtype=torch.float32).pin_memory()
    e2e_steps = 0 if args.no_e2e else max(10, min(args.steps, 500))

    def e2e_step():
        if rg is not None:  # host x in, the fused all-gather matvec, every row's logit into pinned host memory
            rg.step_hostio(wp, rows_per, K, C.c_void_p(xh.data_ptr()), C.c_void_p(xd.data_ptr()), r0,
                           C.c_void_p(lh.data_ptr()), sp, TY)
            return
        A.check(L.arcllm_cuda_matvec_hostio(TY, wp, rows_per, K, C.c_void_p(xh.data_ptr()),
                                            C.c_void_p(xd.data_ptr()), yp, C.c_void_p(yh.data_ptr()), sp),
                "matvec_hostio")
        if dist is not None:
            dist.all_gather_into_tensor(logits, y)
            lh.copy_(logits, non_blocking=True)
            torch.cuda.current_stream().synchronize()

    for _ in range(3 if e2e_steps else 0):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / max(1, e2e_steps)
    if dist is not None:
        tt = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt[0])
    e2e_val = alg_total / (e2e_ms * 1e-3) / 1e9
    d2h = 4 * rows_per * world
    if not e2e_steps:
        e2e_val = None

    extra = {}
    if world == 1 and headline and not args.no_extra:
        extra = run_extra(A, L, torch, dev, sp, hbm_peak)
    if world > 1 and headline:
        # every rank's gathered logits against the single-GPU matvec of the whole head (447 MB, filled here)
        wf = torch.empty(ROWS * rb + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_" + fmt, C.c_void_p(wf.data_ptr()), 0, ROWS * (K // 256), 0x1A4D, sp)
        yf = torch.empty(ROWS, dtype=torch.float32, device=dev)
        A.check(L.arcllm_cuda_matvec(TY, C.c_void_p(wf.data_ptr()), ROWS, K, xp, None, C.c_float(0.0), None, None,
                                     C.c_void_p(yf.data_ptr()), sp), "matvec")
        if rg is not None:
            got = torch.empty(ROWS, dtype=torch.float32, device=dev)
            A.check(L.arcllm_cuda_memcpy_d2h(C.c_void_p(lh.data_ptr()), C.c_void_p(rg.logits_ptr), 4 * ROWS, sp))
            A.check(L.arcllm_cuda_stream_synchronize(sp))
            got.copy_(lh)
        else:
            got = logits
        torch.cuda.synchronize()
        same = torch.tensor([int(torch.equal(got.view(torch.int32), yf.view(torch.int32)))], device=dev)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        extra["gather_bit_exact"] = bool(same.item())
        del wf, yf
        torch.cuda.empty_cache()
        if not args.no_extra:
            extra.update(run_extra_multi(A, L, torch, dist, dev, sp, world, rank, hbm_peak, barrier))

    if rank == 0:
        cpu = None if args.no_cpu or world > 1 or not headline else cpu_baseline()
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {
                "workload": ("config1: Q6_K LM-head matvec 152064x3584 (447.07 MB packed weights), fp32 x ~ N(0,1)"
                             if headline else "profiling case: %s matvec %dx%d" % (fmt, ROWS, K))
                            + (("; rows sharded over %d GPUs, fp32 logits all-gathered by the matvec kernel itself "
                                "(NVLink peer stores of epoch-tagged 64-bit words)" % world if rg is not None else
                                "; rows sharded over %d GPUs + NCCL all-gather of fp32 logits" % world)
                               if world > 1 else ""),
                "l2": "weights larger than L2 (%.0f MB vs 126 MB): no flush needed between steps"
                      % (q_bytes(fmt, ROWS, K) / 1e6),
                "parallelism": "row-shard%d" % world,
                "algorithmic_bytes_per_step": alg_total,
            },
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                "kernel": "matvec_imma_kernel (%s)" % fmt + (" with the NVLink all-gather epilogue; kernel_ms "
                                                             "includes the peer stores and the wait for every rank's rows"
                                                             if rg is not None else ""),
                "kernel_ms": round(kern_ms, 5), "peak_source": peak_src + " (MEASURED_PEAKS.json hbm_gbs, burst copy)",
                "timing": ("mean launch time over one CUDA-graph replay of the %d timed launches%s" %
                           (args.steps, "" if not overlap else ", consecutive launches overlapping (programmatic "
                            "dependent launch)")
                           if args.launch == "graph" and (world == 1 or rg is not None) else
                           "CUDA events around each launch on its stream, mean over the timed launches"),
            },
            "e2e": {"value": None if e2e_val is None else round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": 4 * K,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
                    "api": ("arcllm_cuda_matvec_allgather_hostio (pinned host x copied in, every rank's logits "
                            "stored by the kernel's collect phase into pinned mapped host memory, stream sync)"
                            if rg is not None else
                            "arcllm_cuda_matvec_hostio (pinned host x copied in, logits stored by the kernel into "
                            "pinned mapped host memory, stream sync)")},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if extra:
            line["extra"] = extra
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()
        if rg is not None:
            dist.barrier()  # every rank's last launch is done before the buffers go away
            rg.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_extra_multi(A, L, torch, dist, dev, sp, world, rank, hbm_peak, barrier):
    """The sharded configurations at N > 1 (every time the max over ranks):
    config 1b (Q6_K FFN down 3584x18944) row-sharded with the rows
    re-assembled on every rank by the NVLink exchange kernel, checked against
    the single-GPU matvec; config 4's gate GEMM (256x18944x3584) with its
    output rows (the weight rows) sharded and the shards all-gathered with
    NCCL; config 3's greedy decode of the Qwen2.5-7B-shaped model with the FFN
    and LM head sharded over the ranks (tensor-parallel generate())."""
    from arcllm_b200.rank_gather import ExchangeBuffers
    out = {}

    def exchange(h):
        res = [None] * world
        dist.all_gather_object(res, h)
        return res

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def shard(n, align=32):
        r0, rows = C.c_uint32(0), C.c_uint32(0)
        A.call("arcllm_cuda_shard_rows", n, align, world, rank, C.byref(r0), C.byref(rows))
        return r0.value, rows.value

    # ---- config 1b: Q6_K 3584 x 18944, rows sharded, exchange-gathered ----
    h0, hr = shard(HIDDEN)
    rb = q_bytes("q6k", 1, FFN)
    ncop = max(2, -(-3 * L2_BYTES // (hr * rb)))
    ws = []
    for c in range(ncop):
        t = torch.empty(hr * rb + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_q6k", C.c_void_p(t.data_ptr()), h0 * (FFN // 256), hr * (FFN // 256), 0x1B00 + c, sp)
        ws.append(t)
    x18 = torch.empty(FFN, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(x18.data_ptr()), 0, FFN, 0x1B77, C.c_float(0), C.c_float(1), sp)
    part = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    full = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    ex = ExchangeBuffers(FFN, world, rank, exchange)
    barrier()

    def step1b(i, stream):
        A.check(L.arcllm_cuda_matvec(A.GGML_Q6_K, C.c_void_p(ws[i % ncop].data_ptr()), hr, FFN,
                                     C.c_void_p(x18.data_ptr()), None, C.c_float(0), None, None,
                                     C.c_void_p(part.data_ptr() + 4 * h0), stream), "matvec")
        ex.gather(C.c_void_p(part.data_ptr() + 4 * h0), hr, h0, C.c_void_p(full.data_ptr()), HIDDEN, stream)

    for i in range(10):
        step1b(i, sp)
    barrier()
    # the timed steps as one CUDA graph (matvec + exchange per step, consecutive launches overlapping);
    # the exchange's sequence numbers live on the device, so the graph replays unchanged
    n_it = 200
    A.check(L.arcllm_cuda_set_launch_overlap(1), "launch overlap")
    g1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1, capture_error_mode="thread_local"):
        cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        for i in range(n_it):
            step1b(i, cs)
    A.check(L.arcllm_cuda_set_launch_overlap(0), "launch overlap")
    g1.replay()  # upload: an untimed pass
    barrier()
    step1b(0, sp)  # rendezvous: its exchange ends on every rank within a flag round trip of the others
    A.check(L.arcllm_cuda_stream_delay_us(2000, sp), "stream_delay")
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g1.replay()
    b.record()
    barrier()
    del g1
    ms = max_over_ranks(a.elapsed_time(b) / n_it)
    # check: the last step used copy (n_it - 1) % ncop; the full matrix of that seed on one GPU
    wf = torch.empty(HIDDEN * rb + 16, dtype=torch.uint8, device=dev)
    A.call("arcllm_cuda_fill_q6k", C.c_void_p(wf.data_ptr()), 0, HIDDEN * (FFN // 256), 0x1B00 + (n_it - 1) % ncop, sp)
    yf = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    A.check(L.arcllm_cuda_matvec(A.GGML_Q6_K, C.c_void_p(wf.data_ptr()), HIDDEN, FFN, C.c_void_p(x18.data_ptr()), None,
                                 C.c_float(0), None, None, C.c_void_p(yf.data_ptr()), sp), "matvec")
    # and every rank's shard rows computed alone on this GPU (the split-K grouping depends on the row
    # count, so only the same rows are expected to agree bit for bit)
    ys = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    for q in range(world):
        q0, qr = C.c_uint32(0), C.c_uint32(0)
        A.call("arcllm_cuda_shard_rows", HIDDEN, 32, world, q, C.byref(q0), C.byref(qr))
        A.check(L.arcllm_cuda_matvec(A.GGML_Q6_K, C.c_void_p(wf.data_ptr() + q0.value * rb), qr.value, FFN,
                                     C.c_void_p(x18.data_ptr()), None, C.c_float(0), None, None,
                                     C.c_void_p(ys.data_ptr() + 4 * q0.value), sp), "matvec")
    torch.cuda.synchronize()
    diff = float((full.double() - yf.double()).norm() / yf.double().norm())
    same_rows = int(torch.equal(full.view(torch.int32), ys.view(torch.int32)))
    alg = matvec_alg_bytes("q6k", HIDDEN, FFN)
    out["config1b_q6k_3584x18944_rowshard"] = {
        "GB/s": round(alg / (ms * 1e-3) / 1e9, 1), "us_per_step": round(ms * 1e3, 2),
        "rows_per_rank": hr, "collective": "exchange kernel (NVLink peer stores of epoch-tagged 64-bit words)",
        "timing": "one CUDA graph of %d steps (matvec + exchange each), after a device rendezvous" % n_it,
        "rel_l2_vs_1gpu": float("%.3g" % max_over_ranks(diff)),
        "bit_exact_vs_1gpu_same_rows": bool(max_over_ranks(-same_rows) == -1)}
    del ws, wf, ys
    torch.cuda.synchronize()
    barrier()
    ex.close()
    torch.cuda.empty_cache()

    # ---- config 4: prefill gate GEMM, output rows sharded; the result all-gathered by the GEMM's
    # split-K reduce kernel over NVLink peer stores (NCCL all-gather timed beside it) ----
    from arcllm_b200.rank_gather import GemmGather
    _, tflops_peak, _ = measured_peaks()
    m = 256
    f0, fr = shard(FFN, 128)
    ncop = max(2, -(-3 * L2_BYTES // q_bytes("q4k", fr, HIDDEN)))
    ws = []
    for c in range(ncop):
        t = torch.empty(q_bytes("q4k", fr, HIDDEN) + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_q4k", C.c_void_p(t.data_ptr()), f0 * (HIDDEN // 256), fr * (HIDDEN // 256),
               0x1C00 + c, sp)
        ws.append(t)
    xf = torch.empty(m * HIDDEN, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(xf.data_ptr()), 0, m * HIDDEN, 0x1C7A, C.c_float(0),
           C.c_float(1), sp)
    xb = xf.to(torch.bfloat16)
    sizes = [None] * world
    dist.all_gather_object(sizes, (f0, fr))
    fmax = max(r_ for _, r_ in sizes)  # NCCL form: shards padded to the largest, one all-gather of equal parts
    y = torch.empty(m * fmax, dtype=torch.float32, device=dev)
    yall = torch.empty(world * m * fmax, dtype=torch.float32, device=dev)
    gg = GemmGather(m, FFN, world, rank, exchange)

    def step4(i):
        gg.step(A.GGML_Q4_K, C.c_void_p(ws[i % ncop].data_ptr()), fr, HIDDEN, C.c_void_p(xb.data_ptr()), f0, sp)

    def step4_nccl(i):
        A.check(L.arcllm_cuda_gemm_q4k_bf16(C.c_void_p(ws[i % ncop].data_ptr()), fr, HIDDEN,
                                            C.c_void_p(xb.data_ptr()), m, C.c_void_p(y.data_ptr()), sp), "gemm")
        dist.all_gather_into_tensor(yall, y)

    def timed4(step, n_it=50):
        for i in range(5):
            step(i)
        barrier()
        # rendezvous (one untimed step: its gather ends on every rank together) and 2 ms of wall-clock
        # delay, for both forms, so the first timed step does not absorb the host skew of the barrier
        step(5)
        A.check(L.arcllm_cuda_stream_delay_us(2000, sp), "stream_delay")
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(n_it):
            step(i)
        b.record()
        barrier()
        return max_over_ranks(a.elapsed_time(b) / n_it), n_it

    ms, n_it = timed4(step4)
    # check: every rank's gathered result against plain single-GPU GEMMs of each rank's shard (same
    # split-K as the shard's own launch, so bit for bit), weights of the last step's copy
    last = (n_it - 1) % ncop
    got_h = torch.empty(m * FFN, dtype=torch.float32).pin_memory()
    A.check(L.arcllm_cuda_memcpy_d2h(C.c_void_p(got_h.data_ptr()), C.c_void_p(gg.y_ptr), 4 * m * FFN, sp), "d2h")
    A.check(L.arcllm_cuda_stream_synchronize(sp), "sync")
    got = got_h.to(dev).view(m, FFN)
    same = 1
    for q0, qr in sizes:
        wq = torch.empty(q_bytes("q4k", qr, HIDDEN) + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_q4k", C.c_void_p(wq.data_ptr()), q0 * (HIDDEN // 256), qr * (HIDDEN // 256),
               0x1C00 + last, sp)
        yq = torch.empty(m * qr, dtype=torch.float32, device=dev)
        A.check(L.arcllm_cuda_gemm_q4k_bf16(C.c_void_p(wq.data_ptr()), qr, HIDDEN, C.c_void_p(xb.data_ptr()), m,
                                            C.c_void_p(yq.data_ptr()), sp), "gemm")
        torch.cuda.synchronize()
        same &= int(torch.equal(got[:, q0:q0 + qr].contiguous().view(torch.int32), yq.view(m, qr).view(torch.int32)))
        del wq, yq
    bits = C.c_uint32(0)
    dev_err = L.arcllm_cuda_device_error(sp, C.byref(bits))
    ms_nccl, _ = timed4(step4_nccl)
    tf = 2.0 * m * FFN * HIDDEN / (ms * 1e-3) / 1e12
    out["config4_prefill_gate_256x18944x3584_rowshard"] = {
        "TFLOP/s": round(tf, 1), "frac_of_bf16_peak_per_gpu": round(tf / world / tflops_peak, 4) if tflops_peak else None,
        "us_per_step": round(ms * 1e3, 2), "rows_per_rank": fr,
        "collective": "fused: the GEMM's split-K reduce kernel stores the shard into every rank's m x 18944 result "
                      "(NVLink peer stores) + flag handshake",
        "bit_exact_vs_1gpu_shards": bool(max_over_ranks(-same) == -1) and dev_err == 0,
        "us_per_step_gemm_plus_nccl_allgather": round(ms_nccl * 1e3, 2)}
    del ws, xf, xb, y, yall, got, got_h
    torch.cuda.synchronize()
    barrier()
    gg.close()
    torch.cuda.empty_cache()
    barrier()

    # ---- config 3: tensor-parallel greedy decode ----
    from arcllm_b200.synthetic import QWEN25_7B, SyntheticModel
    md = SyntheticModel(QWEN25_7B, seed=0xC3)
    exd = ExchangeBuffers(md.tp_exchange_words(world), world, rank, exchange)
    md.set_tensor_parallel(exd.ptrs, world, rank)
    barrier()
    prompt = [int(splitmix_token(i, QWEN25_7B["vocab"])) for i in range(256)]
    md.generate(prompt[:8], 4)  # warm-up: captures the step graphs
    barrier()
    t0 = time.perf_counter()
    toks, st = md.generate(prompt, 128)
    wall = time.perf_counter() - t0
    dec_ms = max_over_ranks(st.decode_ms)
    pf_ms = max_over_ranks(st.prefill_ms)
    same = [None] * world
    dist.all_gather_object(same, toks)
    tps = st.decode_steps / (dec_ms * 1e-3)
    bpt = md.bytes_per_token()
    out["config3_decode_tp"] = {
        "tok/s": round(tps, 1), "ms_per_token": round(dec_ms / st.decode_steps, 4),
        "weight_GB/s_whole_job": round(bpt * tps / 1e9, 1), "prefill_ms_256_tokens": round(pf_ms, 2),
        "e2e_generate_s": round(max_over_ranks(wall), 4), "launches_per_token": st.decode_launches_per_step,
        "ranks_agree": all(t == toks for t in same), "first_tokens": toks[:4],
        "sharding": "FFN gate/up rows and the same K window of the FFN down projection over %d ranks (down "
                    "partials all-reduced by the NVLink exchange kernel), LM-head rows sharded (greedy records "
                    "exchanged); attention replicated" % world}
    torch.cuda.synchronize()
    barrier()
    md.close()
    exd.close()
    torch.cuda.empty_cache()
    # the 1-GPU tokens of the same request, on rank 0 (after the ranks are done with NVLink)
    if rank == 0:
        m1 = SyntheticModel(QWEN25_7B, seed=0xC3)
        out["config3_decode_tp"]["tokens_equal_1gpu"] = m1.generate(prompt, 128)[0] == toks
        m1.close()
        torch.cuda.empty_cache()
    barrier()
    return out


def run_extra(A, L, torch, dev, sp, hbm_peak, which="all"):
    """Configs 0, 1b and 2 at N=1 (each timed over rotating weight copies whose
    total exceeds 3x L2; 200 launches after 10 warm-ups, captured in one CUDA
    graph and timed with CUDA events)."""
    out = {}

    def timed(launch, n_iter=200, warm=10):
        """Device time per launch: the n_iter launches are captured into one
        CUDA graph (so host launch overhead does not gap the stream), with
        consecutive launches overlapping as in the headline (programmatic
        dependent launch: a launch streams its weights while its predecessor
        drains, then waits for it before reading inputs or writing outputs),
        and the graph replay is timed with CUDA events on its stream."""
        for i in range(warm):
            launch(i, sp)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        A.check(L.arcllm_cuda_set_launch_overlap(1), "launch overlap")
        try:
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
                for i in range(n_iter):
                    launch(i, cs)
        finally:
            A.check(L.arcllm_cuda_set_launch_overlap(0), "launch overlap")
        g.replay()  # warm replay
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) / n_iter

    def copies(nbytes):
        return max(2, -(-3 * L2_BYTES // nbytes))

    def make_w(fmt, rows, k, n, seed):
        nb = k // 256
        ws = []
        for c in range(n):
            t = torch.empty(q_bytes(fmt, rows, k) + 16, dtype=torch.uint8, device=dev)
            A.call("arcllm_cuda_fill_" + fmt, C.c_void_p(t.data_ptr()), 0, rows * nb, seed + c, sp)
            ws.append(t)
        return ws

    if which == "prefill":
        return run_prefill_gemm(A, L, torch, dev, sp, timed, copies, make_w)

    x18 = torch.empty(FFN, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(x18.data_ptr()), 0, FFN, 0x77, C.c_float(0), C.c_float(1), sp)
    x35 = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(x35.data_ptr()), 0, HIDDEN, 0x78, C.c_float(0), C.c_float(1), sp)
    y18 = torch.empty(FFN, dtype=torch.float32, device=dev)
    y35 = torch.empty(HIDDEN, dtype=torch.float32, device=dev)

    for name, fmt, rows, k, xv, yv in (("config0_q4k_18944x3584", "q4k", FFN, HIDDEN, x35, y18),
                                       ("config1b_q6k_3584x18944", "q6k", HIDDEN, FFN, x18, y35),
                                       ("q4k_3584x18944", "q4k", HIDDEN, FFN, x18, y35)):
        n = copies(q_bytes(fmt, rows, k))
        ws = make_w(fmt, rows, k, n, 0x100)
        ty = A.GGML_Q4_K if fmt == "q4k" else A.GGML_Q6_K

        def launch(i, stream, ws=ws, ty=ty, rows=rows, k=k, xv=xv, yv=yv):
            st = L.arcllm_cuda_matvec(ty, C.c_void_p(ws[i % len(ws)].data_ptr()), rows, k, C.c_void_p(xv.data_ptr()),
                                      None, C.c_float(0), None, None, C.c_void_p(yv.data_ptr()), stream)
            if st:
                A.check(st, name)

        ms = timed(launch)
        gbs = matvec_alg_bytes(fmt, rows, k) / (ms * 1e-3) / 1e9
        out[name] = {"GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 4), "us": round(ms * 1e3, 2),
                     "weight_copies": n}
        del ws
        torch.cuda.empty_cache()

    # route B of the Q4 FFN-down capability: the EXEC148 image of Q4_K 3584x18944
    n = copies(HIDDEN * (FFN // 256) * 148)
    src = make_w("q4k", HIDDEN, FFN, n, 0x100)
    imgs = []
    for t in src:
        img = torch.empty(HIDDEN * (FFN // 256) * 148 + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_exec148_materialize", C.c_void_p(t.data_ptr()), HIDDEN * (FFN // 256),
               C.c_void_p(img.data_ptr()), sp)
        imgs.append(img)
    del src

    def launch_b(i, stream):
        A.check(L.arcllm_cuda_matvec(A.TYPE_EXEC148, C.c_void_p(imgs[i % len(imgs)].data_ptr()), HIDDEN, FFN,
                                     C.c_void_p(x18.data_ptr()), None, C.c_float(0), None, None,
                                     C.c_void_p(y35.data_ptr()), stream), "exec148")

    ms = timed(launch_b)
    alg = HIDDEN * (FFN // 256) * 148 + 4 * (FFN + HIDDEN)
    out["q4k_down_route_b_exec148_3584x18944"] = {"GB/s": round(alg / (ms * 1e-3) / 1e9, 1),
                                                   "frac_of_hbm": round(alg / (ms * 1e-3) / 1e9 / hbm_peak, 4),
                                                   "us": round(ms * 1e3, 2), "weight_copies": n}
    del imgs
    torch.cuda.empty_cache()

    # config 2: one FFN block (RMSNorm -> fused gate/up + SiLU -> down + residual), all Q4_K
    n = copies(3 * q_bytes("q4k", FFN, HIDDEN))
    wg = make_w("q4k", FFN, HIDDEN, n, 0x200)
    wu = make_w("q4k", FFN, HIDDEN, n, 0x300)
    wd = make_w("q4k", HIDDEN, FFN, n, 0x400)
    gamma = torch.empty(HIDDEN, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(gamma.data_ptr()), 0, HIDDEN, 0x79, C.c_float(1), C.c_float(0.1),
           sp)
    s = torch.empty(FFN, dtype=torch.float32, device=dev)
    h = torch.empty(HIDDEN, dtype=torch.float32, device=dev)

    def ffn(i, stream):  # RMSNorm + gate/up + SiLU*up, then down + residual (two launches)
        c = i % n
        A.check(L.arcllm_cuda_ffn_block(A.GGML_Q4_K, C.c_void_p(wg[c].data_ptr()), C.c_void_p(wu[c].data_ptr()),
                                        C.c_void_p(wd[c].data_ptr()), HIDDEN, FFN, C.c_void_p(x35.data_ptr()),
                                        C.c_void_p(gamma.data_ptr()), C.c_float(1e-6), C.c_void_p(s.data_ptr()),
                                        C.c_void_p(x35.data_ptr()), C.c_void_p(h.data_ptr()), stream), "ffn block")

    ms = timed(ffn, n_iter=100)
    alg = 3 * q_bytes("q4k", FFN, HIDDEN) + 4 * (HIDDEN * 3 + FFN * 2)
    out["config2_ffn_block_q4k"] = {"GB/s": round(alg / (ms * 1e-3) / 1e9, 1),
                                    "frac_of_hbm": round(alg / (ms * 1e-3) / 1e9 / hbm_peak, 4),
                                    "us": round(ms * 1e3, 2), "launches": 2, "api": "arcllm_cuda_ffn_block"}
    del wg, wu, wd
    torch.cuda.empty_cache()
    out.update(run_prefill_gemm(A, L, torch, dev, sp, timed, copies, make_w))
    out["config3_decode"] = run_decode(A, torch, hbm_peak)
    return out


def run_one_matvec(A, torch, hbm_peak, fmt, rows, k, steps, warmup, dual=False):
    """One matvec shape (or the fused Q4_K gate/up pair with RMSNorm and
    SiLU*mul when `dual`) launched `steps` times on one stream over rotating
    weight copies totalling >= 3x L2, timed with CUDA events around the whole
    run (for launch lists and single-kernel ncu captures)."""
    dev = torch.device("cuda", 0)
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = A.lib()
    if dual:
        fmt = "q4k"
    nmat = 2 if dual else 1
    per = nmat * q_bytes(fmt, rows, k)
    ncop = max(2, -(-3 * L2_BYTES // per))
    ws = []
    for c in range(ncop * nmat):
        t = torch.empty(q_bytes(fmt, rows, k) + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_" + fmt, C.c_void_p(t.data_ptr()), 0, rows * (k // 256), 0x600 + c, sp)
        ws.append(t)
    x = torch.empty(k, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(x.data_ptr()), 0, k, 0x7B, C.c_float(0), C.c_float(1), sp)
    gamma = torch.empty(k, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(gamma.data_ptr()), 0, k, 0x7C, C.c_float(1), C.c_float(0.1), sp)
    y = torch.empty(rows, dtype=torch.float32, device=dev)
    ty = A.GGML_Q4_K if fmt == "q4k" else A.GGML_Q6_K

    def launch(i):
        c = i % ncop
        if dual:
            A.check(L.arcllm_cuda_gateup_silu_q4k(C.c_void_p(ws[2 * c].data_ptr()), C.c_void_p(ws[2 * c + 1].data_ptr()),
                                                  rows, k, C.c_void_p(x.data_ptr()), C.c_void_p(gamma.data_ptr()),
                                                  C.c_float(1e-6), C.c_void_p(y.data_ptr()), sp), "gateup")
        else:
            A.check(L.arcllm_cuda_matvec(ty, C.c_void_p(ws[c].data_ptr()), rows, k, C.c_void_p(x.data_ptr()), None,
                                         C.c_float(0), None, None, C.c_void_p(y.data_ptr()), sp), "matvec")

    for i in range(warmup):
        launch(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        launch(i)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / max(1, steps)
    alg = nmat * q_bytes(fmt, rows, k) + 4 * (k + rows)
    return {"workload": ("gateup_q4k_2x%dx%d" % (rows, k)) if dual else ("%s_%dx%d" % (fmt, rows, k)),
            "us_per_launch_stream": round(ms * 1e3, 2), "GB/s": round(alg / (ms * 1e-3) / 1e9, 1),
            "frac_of_hbm": round(alg / (ms * 1e-3) / 1e9 / hbm_peak, 4), "weight_copies": ncop, "launches": steps}


def run_prefill_gemm(A, L, torch, dev, sp, timed, copies, make_w, m=256):
    """Config 4: the prefill GEMMs at M=256 prompt tokens on tcgen05 (bf16 x,
    Q4_K weights dequantised to bf16 on chip, fp32 accumulation), over rotating
    weight copies; TFLOP/s against the measured bf16 peak."""
    _, tflops_peak, _ = measured_peaks()
    out = {}
    xf = torch.empty(m * FFN, dtype=torch.float32, device=dev)  # seeded N(0,1) activations, as bf16
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(xf.data_ptr()), 0, m * FFN, 0x7A, C.c_float(0), C.c_float(1), sp)
    x = xf.to(torch.bfloat16)
    for name, n, k in (("config4_prefill_gate_256x18944x3584", FFN, HIDDEN),
                       ("config4_prefill_down_256x3584x18944", HIDDEN, FFN)):
        nc = copies(q_bytes("q4k", n, k))
        ws = make_w("q4k", n, k, nc, 0x500)
        y = torch.empty(m, n, dtype=torch.float32, device=dev)

        def launch(i, stream, ws=ws, n=n, k=k, y=y):
            A.check(L.arcllm_cuda_gemm_q4k_bf16(C.c_void_p(ws[i % len(ws)].data_ptr()), n, k,
                                                C.c_void_p(x.data_ptr()), m, C.c_void_p(y.data_ptr()), stream),
                    "gemm")

        ms = timed(launch, n_iter=50)
        tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
        out[name] = {"TFLOP/s": round(tf, 1), "frac_of_bf16_peak": round(tf / tflops_peak, 4) if tflops_peak else None,
                     "us": round(ms * 1e3, 2), "weight_copies": nc}
        del ws
        torch.cuda.empty_cache()
    return out


def run_decode(A, torch, hbm_peak, n_prompt=256, max_new=128):
    """Config 3: greedy decode of a random-init Qwen2.5-7B-shaped model (q/k/o/
    gate/up Q4_K; v, down, LM head Q6_K; fp16 embedding; fp16 KV cache, max
    context 4096): 256 seeded uniform prompt ids, then 128 greedy tokens, one
    CUDA-graph launch per token, the next token chosen on the device."""
    from arcllm_b200.synthetic import QWEN25_7B, SyntheticModel
    m = SyntheticModel(QWEN25_7B, seed=0xC3)
    prompt = [int(splitmix_token(i, QWEN25_7B["vocab"])) for i in range(n_prompt)]
    m.generate(prompt[:min(8, n_prompt)], 4)  # warm-up: captures the two step graphs
    t0 = time.perf_counter()
    toks, st = m.generate(prompt, max_new)
    wall = time.perf_counter() - t0
    bpt = m.bytes_per_token()
    dec_s = st.decode_ms * 1e-3
    tps = st.decode_steps / dec_s
    res = {"tok/s": round(tps, 1), "ms_per_token": round(st.decode_ms / st.decode_steps, 4),
           "weight_GB/s": round(bpt * tps / 1e9, 1), "frac_of_hbm": round(bpt * tps / 1e9 / hbm_peak, 4),
           "bytes_per_token": bpt, "prefill_ms_256_tokens": round(st.prefill_ms, 2),
           "e2e_generate_s": round(wall, 4),
           "e2e_tok_s_incl_prefill": round(max_new / wall, 1),
           "launches_per_token": st.decode_launches_per_step, "graph_launches_per_token": 1,
           "first_tokens": toks[:4], "finite": bool(st.finite)}
    # Precision of the default path (batched bf16 tensor-core prefill) against the fp32
    # token-by-token prefill on the same prompt, both on this GPU (the CPU-oracle check of
    # the 28-layer model is tests/test_decode_e2e_gpu.py): the generated tokens position by
    # position, and the logits of the first decode steps.
    m.set_prefill_mode(0)
    toks32, _ = m.generate(prompt, max_new)
    window = min(4, max_new)
    lg = {}
    for mode in (1, 0):
        m.set_prefill_mode(mode)
        m.begin(prompt, window)
        m.prefill()
        lg[mode] = []
        for _ in range(window):
            m.step(with_head=True, use_graph=True)
            lg[mode].append(m.logits().astype("float64"))
    import numpy as np
    rels = [float(np.linalg.norm(a - b) / np.linalg.norm(b)) for a, b in zip(lg[1], lg[0])]
    res["vs_fp32_token_prefill"] = {
        "token_match_rate": round(sum(int(a == b) for a, b in zip(toks, toks32)) / max_new, 4),
        "logits_rel_l2_max_first_%d_steps" % window: float("%.3g" % max(rels))}
    m.close()
    torch.cuda.empty_cache()
    return res


def splitmix_token(i, vocab, seed=0x70C):
    from arcllm_b200.synthetic import splitmix64_at
    return ((splitmix64_at(seed, i) >> 32) * vocab) >> 32


if __name__ == "__main__":
    sys.exit(main())
