"""Benchmark: draft-tree cycles/sec at batch 64 per GPU (score + build + GDN
verify + commit), with roofline, CPU baseline and end-to-end numbers.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one full cycle over the batch (see dforktree_b200/cycle.py):
score+build of 64 requests (S=24 positions over V=248,320 fp32 logits, the
config-0 n-gram table shared), tree conv + GDN tree verify on each of the 24
GDN layers of the Qwen3.5-9B shape (Hk=16, Hv=32, D=128), greedy tree
acceptance against a target stand-in that agrees with the draft along the
deepest node's path for a drawn length U[1,24] (cut at the path's end), and
the closed-form commit of every layer's state.  Data is synthetic (seeded;
random-init layer weights).  Under torchrun every rank runs its own batch of
64 requests (weak scaling, no collective on the data path); timing is CUDA
events on each rank, the maximum over ranks.

The line also carries `config4`: BASELINE config 4 -- 256 requests split over
the ranks (strong scaling), the hybrid 32-layer stack with the 8 gated
attention layers inside the cycle, chain-first trees with accepted lengths
U[1,24].  `--impl reference` times whole cycles of the reference on the host
cores and, in a child process, the reference's own Triton / torch GPU path
(`reference_gpu`).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "draft-tree cycles/sec (score+build+GDN verify+commit) at batch 64; % roofline"
WORKLOAD = ("dforktree cycle (BASELINE config 1 + GDN verify/commit): batch 64/GPU, S=24, V=248320 fp32 logits, "
            "2M+8M n-gram table, B=32 nodes, M=16, 24 Qwen3.5-9B GDN layers (tree conv + verify, Hk=16 Hv=32 "
            "D=128, bf16 activations, fp32 state), greedy accept along the deepest node's path (drawn length "
            "U[1,24], cut at the path's end), in-place commit")
S, V, N, M, LAYERS, HK, HV, D = 24, 248320, 32, 16, 24, 16, 32, 128
C_CONV = 2 * HK * D + HV * D
# algorithmic bytes per unit (per layer-request): state in, q / k / v in, gates, o out
VERIFY_BYTES = 2 * 1024 * 1024 + 262144 + 262144 + 8192 + 262144      # S0 + q,k + v + g,beta + o
# the fused launch also reads the conv state / weights and writes the aux rows the commit needs
VERIFY_AUX_BYTES = 8192 * 3 * 2 + 262144 + 524288 + 4096               # conv state + k_hat + vn + G
# the plugin's default tree of 64 nodes (fc1_fused.py:4): q / k / v, gates and o double
VERIFY_BYTES_N64 = 2 * 1024 * 1024 + 2 * (262144 + 262144 + 8192 + 262144)
COMMIT_BYTES_FIXED = 4 * 1024 * 1024                                   # read S0 + write S
COMMIT_BYTES_PER_NODE = 32 * 1024                                      # k, vn rows of 32 heads
SCORE_BYTES = S * V * 4 + 105984 * 12 + 2944                           # logits + table probes + prev/pn
# gated full-attention layers (config 3): 16 q-heads / 4 kv-heads at dim 256, 4K-token prefix + the tree
ATTN_HQ, ATTN_HKV, ATTN_D, ATTN_PREFIX = 16, 4, 256, 4096
ATTN_KEYS = ATTN_PREFIX + N
# per layer-request: K and V of every key (bf16), q and o (bf16), the key slot indices (int32)
ATTN_BYTES = ATTN_KEYS * ATTN_HKV * ATTN_D * 2 * 2 + 2 * N * ATTN_HQ * ATTN_D * 2 + ATTN_KEYS * 4
ATTN_FLOPS = 4 * N * ATTN_HQ * ATTN_KEYS * ATTN_D


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# --------------------------------------------------------- CPU baseline ----
def _ref_dir():
    """The reference's dforktree/ sources as installed under baseline/_ref
    (pip install --target; travels with the tree), or None."""
    d = os.path.join(ROOT, "baseline", "_ref", "dforktree")
    return d if os.path.isfile(os.path.join(d, "fc1_builder.py")) else None


_W = {}    # per-worker state of the CPU pool


def _cpu_init(tdir, npz, ref_dir, n_logits, n_layers):
    """Worker set-up (spawned, single-threaded): the n-gram table, a few
    request inputs, and the builder -- the reference's own torch code when its
    sources are installed, else the numpy port."""
    for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[k] = "1"
    import multiprocessing as mp

    import numpy as np
    from dforktree_b200 import synth
    wid = (mp.current_process()._identity or (0,))[0]
    _W["logits"] = [synth.make_logits(S, V, seed=7000 + 97 * wid + i) for i in range(n_logits)]
    _W["layers"] = [_layer_inputs(9000 + 97 * wid + i) for i in range(n_layers)]
    if ref_dir:
        import torch
        torch.set_num_threads(1)
        from oracle import reference_shim as RS
        mods = RS.load_reference(ref_dir, kernels=False)
        RS.patch_path_fn(mods)
        ng = mods["ngram_gpu"].NGramGPU(npz, "cpu", beta3=60.0)       # fc1_builder.py:17
        _W["builder"] = RS.cpu_builder(mods, ng, S, N)
        _W["torch"] = torch
    else:
        from oracle import ngram as ON
        table = {k[:-4]: np.load(os.path.join(tdir, k), mmap_mode="r") for k in os.listdir(tdir) if k.endswith(".npy")}
        _W["ng"] = ON.NGramOracle(table, beta3=60.0)


def _layer_inputs(seed):
    import numpy as np
    from dforktree_b200 import synth
    d = synth.make_gdn_inputs(N, HK, HV, D, seed=seed)
    rng = np.random.default_rng(seed)
    d["x"] = rng.standard_normal((N, C_CONV)).astype(np.float32)
    d["cs"] = rng.standard_normal((C_CONV, 3)).astype(np.float32)
    d["w"] = rng.standard_normal((C_CONV, 4)).astype(np.float32)
    return d


def _cpu_job(job):
    """One unit of a cycle on the host: a request's score+build ("b") or a
    layer-request's tree conv + GDN verify + closed-form commit ("l")."""
    kind, i = job
    if kind == "b":
        lg = _W["logits"][i % len(_W["logits"])]
        if "builder" in _W:
            torch = _W["torch"]
            b = _W["builder"]
            b.logits = torch.from_numpy(lg)
            b.root.fill_(5)
            b.pre1.fill_(7)
            b.run()                                                     # fc1_builder.py:26-47
        else:
            from oracle import builder as OB
            OB.builder_run(lg, 5, 7, _W["ng"], N=N)
        return kind
    from oracle import builder as OB
    from oracle import gdn as OG
    d = _W["layers"][i % len(_W["layers"])]
    _, _, cidx = OB.tree_struct(d["parent"], 4)
    OG.tree_conv(d["x"], d["cs"], d["w"], None, cidx)
    _, k, vn, G = OG.tree_gdn(d["y"], d["a"], d["b"], d["A_log"], d["dt_bias"], d["pool"], 0, d["anc"], HK, HV, D, D)
    u = int(d["path"][-1])
    for h in range(HV):
        OG.snapshot(d["pool"][0, h], k[h], vn[h], G[h], d["anc"], d["path"], u)
    return kind


class CpuCycle:
    """The cycle on the host cores, whole cycles at a time: a spawn pool of
    `workers` single-threaded processes runs every unit of one batch-64 cycle
    (64 score+builds and 64 x 24 layer-request conv+verify+commits) per
    `cycle()`, timed by wall clock from the first job to the last result.
    Score+build is the reference's own torch code (fc1_builder / tree_ops /
    ngram_gpu from its installed sources, the missing path closure supplied);
    the GDN conv / verify / commit, which the reference has only as Triton
    kernels, run as the numpy port of those kernels."""

    def __init__(self, workers: int, batch: int = 64, layers: int = LAYERS):
        import multiprocessing as mp

        import numpy as np

        from dforktree_b200 import synth
        self.workers, self.batch, self.layers = workers, batch, layers
        self.ref_dir = _ref_dir()
        table = synth.make_ngram_table(V, 2_000_000, 8_000_000, seed=0)
        self.tdir = tempfile.mkdtemp(prefix="dft_table_")
        self.npz = os.path.join(self.tdir, "table.npz")
        if self.ref_dir:
            np.savez(self.npz, **table)
        else:
            for k, v in table.items():
                np.save(os.path.join(self.tdir, k + ".npy"), np.asarray(v))
        del table
        self.pool = mp.get_context("spawn").Pool(workers, initializer=_cpu_init,
                                                 initargs=(self.tdir, self.npz, self.ref_dir, 2, 2))
        # one pass of every job kind on every worker before any timing
        self.pool.map(_cpu_job, [("b", i) for i in range(workers)] + [("l", i) for i in range(workers)], chunksize=1)

    @property
    def kind(self):
        # the GDN stages (most of the time) always run as the port
        return "port"

    def describe(self):
        who = ("the reference's own torch builder (fc1_builder / tree_ops / ngram_gpu, installed sources, "
               "missing path closure supplied)" if self.ref_dir else "the numpy port of the builder")
        return (f"whole cycles: {self.batch} score+builds by {who} and {self.batch} x {self.layers} layer-request "
                f"conv+verify+commits by the numpy port of the reference's Triton kernels, per step, on "
                f"{self.workers} single-threaded processes (wall clock)")

    def cycle(self) -> float:
        jobs = [("b", i) for i in range(self.batch)] + [("l", i) for i in range(self.batch * self.layers)]
        t = time.perf_counter()
        self.pool.map(_cpu_job, jobs, chunksize=8)
        return time.perf_counter() - t

    def close(self):
        self.pool.close()
        self.pool.join()
        for f in os.listdir(self.tdir):
            os.unlink(os.path.join(self.tdir, f))
        os.rmdir(self.tdir)


# ------------------------------------------------------------- clocks ------
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, sampled every 20 ms
    in a background thread through NVML (read-only queries), for the duration of
    the timed region; the GPU is identified by its UUID, so the sample follows
    the device this process runs on whatever CUDA_VISIBLE_DEVICES maps.  Falls
    back to `nvidia-smi -i <uuid>` when NVML is unavailable."""

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.rows = []          # (sm_mhz, max_mhz, set of reasons)
        self._stop = None
        self._thread = None

    def _uuid(self):
        import torch
        u = str(torch.cuda.get_device_properties(self.device_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self._uuid())
            bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}

            def sample():
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(sm), float(mx), {k for k, b in bits.items() if r & b}))
        except Exception:
            sample = self._smi_sampler()

        def loop():
            while not self._stop.is_set():
                try:
                    sample()
                except Exception:
                    pass
                self._stop.wait(0.02)

        if sample is not None:
            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        return self

    def _smi_sampler(self):
        try:
            uuid = self._uuid()
        except Exception:
            return None
        fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

        def sample():
            out = subprocess.run(["nvidia-smi", "-i", uuid, f"--query-gpu={fields}", "--format=csv,noheader,nounits"],
                                 capture_output=True, text=True, timeout=5).stdout.strip().split(",")
            out = [x.strip() for x in out]
            self.rows.append((float(out[0]), float(out[1]),
                              {names[i] for i in range(4) if out[2 + i].lower() == "active"}))
        return sample

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.rows:
            return None
        sm = [r[0] for r in self.rows]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted(set().union(*[r[2] for r in self.rows])), "samples": len(self.rows)}


# ---------------------------------------------------------------- ours -----
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from dforktree_b200 import build as B
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    from dforktree_b200 import workload as WL
    from dforktree_b200.cycle import CycleConfig, DraftTreeCycle

    if rank == 0:
        B.build()
    if world > 1:
        dist.barrier()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = CycleConfig(B=args.batch, layers=args.layers)
    table_np = synth.make_ngram_table(V, 2_000_000, 8_000_000, seed=0)
    from dforktree_b200.ngram_gpu import load_npz_arrays
    table = K.Table(load_npz_arrays(table_np), beta3=60.0, device=dev)
    del table_np
    # config 4 first: its buffers (~63 GB at 256 requests on one GPU) are freed before the headline's
    c4 = _bench_config4(args, rank, world, dev, table) if args.requests > 0 and not args.profile else None
    cyc = DraftTreeCycle(cfg, table, dev, seed=rank)
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + rank)
    Bt = cfg.B
    # synthetic per-step inputs, resident in HBM (larger than L2: no flush needed)
    inp = WL.cycle_inputs(cfg, dev, seed=1234 + rank)
    logits, root, pre1, x, a, b = (inp[k] for k in ("logits", "root", "pre1", "x", "a", "b"))
    acc_len = inp["acc_len"]

    def target_eager(tree):
        # target-model stand-in: agrees with the draft along the deepest node's path up to the drawn length
        return WL.path_target(tree, acc_len)

    stream = torch.cuda.current_stream(dev)
    # the stand-in's ~12 small torch launches replay as one CUDA graph once
    # captured (after the first warm-up step); it reads the cycle's persistent
    # tree buffers, so every replay sees the current tree
    tgt = {"fn": target_eager}

    def target_fn(tree):
        return tgt["fn"](tree)

    def capture_target():
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                target_eager(cyc.tree)
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = target_eager(cyc.tree)
        torch.cuda.synchronize()

        def replay(tree):
            assert tree is cyc.tree
            graph.replay()
            return out
        tgt["fn"] = replay
        tgt["graph"] = graph

    def one_step(ev=None):
        if ev is None:
            cyc.step(logits, root, pre1, x, a, b, target_fn)
            return
        ev["sb0"].record(stream)
        cyc.build(logits, root, pre1)
        ev["sb1"].record(stream)
        for l in range(cfg.layers):
            cyc.verify_layer(l, x[l], a[l], b[l])
        ev["v1"].record(stream)
        cyc.accept(target_fn(cyc.tree))
        ev["c0"].record(stream)
        cyc.commit(x)
        ev["c1"].record(stream)

    for i in range(args.warmup):
        one_step()
        if i == 0:
            capture_target()
    torch.cuda.synchronize()
    if args.profile:
        # profiling mode: just K plain cycles after the warm-up (for ncu)
        for _ in range(args.steps):
            one_step()
        torch.cuda.synchronize()
        return None
    mk = lambda: torch.cuda.Event(enable_timing=True)
    # each verify launch alone (events around every launch: no overlap with the
    # previous layer's launch), reported beside the in-cycle average
    verify_ms = 0.0
    pairs = []
    for _ in range(args.steps):
        cyc.build(logits, root, pre1)
        for l in range(cfg.layers):
            e1, e2 = mk(), mk()
            e1.record(stream)
            cyc.verify_layer(l, x[l], a[l], b[l])
            e2.record(stream)
            pairs.append((e1, e2))
        cyc.accept(target_fn(cyc.tree))
        cyc.commit(x)
    torch.cuda.synchronize()
    for e1, e2 in pairs:
        verify_ms += e1.elapsed_time(e2)
    n_verify = len(pairs)

    # ---- timed region: exactly K steps, barrier + sync on both sides
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = mk(), mk()
    # stage markers inside the timed steps (events between stages: the work and
    # the launch order are those of DraftTreeCycle.step)
    evs = [{k: mk() for k in ("sb0", "sb1", "v1", "c0", "c1")} for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        t0.record(stream)
        for ev in evs:
            one_step(ev)
        t1.record(stream)
        torch.cuda.synchronize()
    stage = {"score_build": 0.0, "conv_verify": 0.0, "accept": 0.0, "commit": 0.0}
    for ev in evs:
        stage["score_build"] += ev["sb0"].elapsed_time(ev["sb1"])
        stage["conv_verify"] += ev["sb1"].elapsed_time(ev["v1"])
        stage["accept"] += ev["v1"].elapsed_time(ev["c0"])
        stage["commit"] += ev["c0"].elapsed_time(ev["c1"])
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    mean_acc = float(cyc.accept_len.float().mean())
    ms_max = ms
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_max = float(tt)
    value = world * args.steps / (ms_max / 1e3)

    # ---- end to end through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        ke = max(1, min(args.steps, 6))
        h_logits = torch.empty(logits.shape, dtype=logits.dtype, pin_memory=True)
        h_x = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        h_a = torch.empty(a.shape, dtype=a.dtype, pin_memory=True)
        h_b = torch.empty(b.shape, dtype=b.dtype, pin_memory=True)
        h_root = torch.empty(root.shape, dtype=root.dtype, pin_memory=True)
        h_pre1 = torch.empty(pre1.shape, dtype=pre1.dtype, pin_memory=True)
        for h, d_ in ((h_logits, logits), (h_x, x), (h_a, a), (h_b, b), (h_root, root), (h_pre1, pre1)):
            h.copy_(d_)
        h_tok = torch.empty((Bt, N), dtype=torch.int64, pin_memory=True)
        h_par = torch.empty((Bt, N), dtype=torch.int64, pin_memory=True)
        h_len = torch.empty((Bt,), dtype=torch.int64, pin_memory=True)
        hosts = (h_logits, h_x, h_a, h_b, h_root, h_pre1)
        # two device copies of the step inputs: step i + 1's are copied on a second
        # stream while step i runs (each buffer is refilled once the step that
        # read it has finished)
        bufs = [tuple(torch.empty_like(t) for t in (logits, x, a, b, root, pre1)) for _ in range(2)]
        cps = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        free = [torch.cuda.Event(), torch.cuda.Event()]
        h2d = sum(t.numel() * t.element_size() for t in hosts)
        d2h = sum(t.numel() * t.element_size() for t in (h_tok, h_par, h_len))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s0, s1 = mk(), mk()

        def issue_copy(i):
            with torch.cuda.stream(cps):
                if i >= 2:
                    cps.wait_event(free[i % 2])
                for d_, h in zip(bufs[i % 2], hosts):
                    d_.copy_(h, non_blocking=True)
                copied[i % 2].record(cps)

        s0.record(stream)
        cps.wait_stream(stream)
        issue_copy(0)
        for i in range(ke):
            if i + 1 < ke:
                issue_copy(i + 1)
            stream.wait_event(copied[i % 2])
            d_logits, d_x, d_a, d_b, d_root, d_pre1 = bufs[i % 2]
            cyc.step(d_logits, d_root, d_pre1, d_x, d_a, d_b, target_fn)
            free[i % 2].record(stream)
            h_tok.copy_(cyc.tree["tokens"], non_blocking=True)
            h_par.copy_(cyc.tree["parent"], non_blocking=True)
            h_len.copy_(cyc.accept_len, non_blocking=True)
        s1.record(stream)
        torch.cuda.synchronize()
        ems = s0.elapsed_time(s1)
        if world > 1:
            tt = torch.tensor([ems], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ems = float(tt)
        e2e = {"value": world * ke / (ems / 1e3), "unit": "cycles/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "steps": ke,
               "pipelined": "step i + 1's inputs copied on a second stream while step i runs"}
    # ---- tree-masked attention verify of one gated full-attention layer (outside the cycle)
    attn = _bench_attention(args, dev, cyc, g, stream) if args.attn else None
    status = int(cyc.status.item())
    # ---- the plugin's default 64-node tree (outside the cycle)
    n64 = _bench_verify_n64(args, dev, table, stream) if args.n64 else None

    if rank != 0:
        return None
    hbm, tflops, peak_kind = _peaks()
    # the dominant kernel's average launch duration over the timed steps (its
    # 24 launches run back to back, each overlapping the previous one's tail)
    verify_launch_ms = stage["conv_verify"] / (args.steps * cfg.layers)
    verify_isolated_ms = verify_ms / max(n_verify, 1)
    commit_launch_ms = stage["commit"] / args.steps
    verify_bytes = Bt * VERIFY_BYTES
    commit_bytes = Bt * LAYERS * (COMMIT_BYTES_FIXED + COMMIT_BYTES_PER_NODE * mean_acc)
    traffic = _traffic()
    cand = {
        "gdn_verify": (verify_launch_ms * LAYERS, verify_bytes, verify_launch_ms),
        "gdn_commit": (commit_launch_ms, commit_bytes, commit_launch_ms),
    }
    dom = max(cand, key=lambda k: cand[k][0])
    _, nbytes, lms = cand[dom]
    achieved = nbytes / (lms / 1e3) / 1e9
    roof = {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": int(nbytes), "launch_ms": round(lms, 4),
            "traffic": traffic.get(dom)}
    per_kernel = {
        "score_build_ms": stage["score_build"] / args.steps,
        "conv_verify_ms_per_layer": verify_launch_ms,
        "conv_verify_isolated_ms_per_layer": verify_isolated_ms,
        "accept_ms": stage["accept"] / args.steps,
        "gdn_commit_ms": commit_launch_ms,
        "score_build_GBps": Bt * SCORE_BYTES / (stage["score_build"] / args.steps / 1e3) / 1e9,
        "gdn_verify_GBps": verify_bytes / (verify_launch_ms / 1e3) / 1e9,
        "gdn_commit_GBps": commit_bytes / (commit_launch_ms / 1e3) / 1e9,
        "mean_accept_len": mean_acc,
        # the whole cycle against the roofline: every stage's algorithmic bytes
        # (score + build, 24 verifies, the commit) over the measured cycle time
        "request_cycles_per_s": Bt * args.steps / (ms / 1e3),
        "cycle_GBps": (Bt * SCORE_BYTES + verify_bytes * cfg.layers + commit_bytes) / (ms / args.steps / 1e3) / 1e9,
    }
    per_kernel["cycle_hbm_frac"] = per_kernel["cycle_GBps"] / hbm
    if attn is not None:
        per_kernel["tree_attn_ms_per_layer"] = attn
        per_kernel["tree_attn_GBps"] = Bt * ATTN_BYTES / (attn / 1e3) / 1e9
        per_kernel["tree_attn_hbm_frac"] = per_kernel["tree_attn_GBps"] / hbm
        per_kernel["tree_attn_TFLOPs"] = Bt * ATTN_FLOPS / (attn / 1e3) / 1e12
    if n64 is not None:
        per_kernel["verify_n64_ms_per_layer"] = n64[0]
        per_kernel["verify_n64_GBps"] = Bt * VERIFY_BYTES_N64 / (n64[0] / 1e3) / 1e9
        per_kernel["verify_n64_hbm_frac"] = per_kernel["verify_n64_GBps"] / hbm
        per_kernel["verify_n64_mean_max_depth"] = n64[1]
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "cycles/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config(Bt, cfg.layers, world),
        "roofline": roof, "stages": {k: round(v, 4) for k, v in per_kernel.items()},
        "gpu_launches": cyc.launches_per_step * args.steps, "dev_status": status,
    }
    if e2e is not None:
        line["e2e"] = e2e
    line["clocks"] = clk.summary()
    if c4 is not None:
        line["config4"] = c4
    return line


CONFIG4 = ("BASELINE config 4 at every N: 256 requests split over the GPUs (strong scaling), each a cycle of "
           "score+build (chain-first trees, so the drawn accepted lengths U[1,24] are reachable) -> 32 Qwen3.5-9B "
           "layers in model order (24 GDN: tree conv + verify; 8 gated attention: tree-masked attention over a "
           "4K-token prefix + the tree, 16 q / 4 kv heads at dim 256) -> greedy accept -> in-place commit")


def _bench_config4(args, rank, world, dev, table):
    """The hybrid-stack cycle of config 4: this rank's share of args.requests,
    W warm-up + K timed cycles (CUDA events, barrier + sync on both sides, max
    over ranks); value = whole-job cycles/s (every cycle covers all requests)."""
    import torch
    import torch.distributed as dist

    from dforktree_b200 import sharding
    from dforktree_b200 import workload as WL
    from dforktree_b200.cycle import CycleConfig, DraftTreeCycle

    shard = sharding.partition(args.requests, world)[rank]
    if shard.count == 0:
        raise SystemExit("config 4: more ranks than requests")
    cfg = CycleConfig(B=shard.count, layers=LAYERS, attn_layers=8, chain_first=True)
    cyc = DraftTreeCycle(cfg, table, dev, seed=100 + rank)
    inp = WL.cycle_inputs(cfg, dev, seed=5678 + rank)
    logits, root, pre1, x, a, b, q = (inp[k] for k in ("logits", "root", "pre1", "x", "a", "b", "q"))
    acc_len = inp["acc_len"]
    stream = torch.cuda.current_stream(dev)
    mk = lambda: torch.cuda.Event(enable_timing=True)

    def one(ev=None):
        if ev is not None:
            ev[0].record(stream)
        cyc.build(logits, root, pre1)
        if ev is not None:
            ev[1].record(stream)
        cyc.verify(x, a, b, q)
        if ev is not None:
            ev[2].record(stream)
        cyc.accept(WL.path_target(cyc.tree, acc_len))
        cyc.commit(x)
        if ev is not None:
            ev[3].record(stream)

    for _ in range(max(args.warmup, 1)):
        one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [[mk() for _ in range(4)] for _ in range(args.steps)]
    t0, t1 = mk(), mk()
    t0.record(stream)
    for ev in evs:
        one(ev)
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    ms_max = ms
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_max = float(tt)
    k = args.steps
    stages = {"score_build_ms": sum(e[0].elapsed_time(e[1]) for e in evs) / k,
              "verify_32_layers_ms": sum(e[1].elapsed_time(e[2]) for e in evs) / k,
              "accept_commit_ms": sum(e[2].elapsed_time(e[3]) for e in evs) / k,
              "mean_accept_len": float(cyc.accept_len.float().mean())}
    status = int(cyc.status.item())
    out = {"workload": CONFIG4, "requests": args.requests, "requests_per_gpu": shard.count,
           "value": round(k / (ms_max / 1e3), 3), "unit": "cycles/s", "ms_per_step": round(ms_max / k, 4),
           "scaling": "strong", "stages": {kk: round(v, 4) for kk, v in stages.items()},
           "gpu_launches": cyc.launches_per_step * k, "dev_status": status}
    del cyc, inp, logits, x, a, b, q
    torch.cuda.empty_cache()
    return out


def _attention_inputs(dev, Bt, anc, g):
    """The attention workload of one gated full-attention layer: 4K-token
    prefixes + the tree in a paged KV cache with shuffled slots (1.1 GB at
    batch 64, larger than L2), planned once."""
    import torch
    from dforktree_b200.tree_attn import TreeAttentionWrapper
    slots = Bt * ATTN_KEYS
    perm = torch.randperm(slots, device=dev, generator=g).to(torch.int32)
    kc = torch.randn(slots, ATTN_HKV, ATTN_D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(slots, ATTN_HKV, ATTN_D, device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn(Bt, N, ATTN_HQ, ATTN_D, device=dev, generator=g).to(torch.bfloat16)
    indptr = (torch.arange(Bt + 1, device=dev) * ATTN_KEYS).to(torch.int32)
    w = TreeAttentionWrapper(dev).plan(indptr, perm, ATTN_HQ, ATTN_HKV, ATTN_D, n=N, anc=anc,
                                       kv_lens_host=[ATTN_KEYS] * Bt)
    return w, q, (kc, vc), torch.empty_like(q)


def _bench_attention(args, dev, cyc, g, stream):
    """Mean CUDA-event time of one tree-masked attention layer (attention +
    split merge) over the batch, the cycle's own trees as masks."""
    import torch
    w, q, kv, o = _attention_inputs(dev, cyc.cfg.B, cyc.tree["anc"], g)
    for _ in range(max(args.warmup, 3)):
        w.run(q, kv, out=o)
    mk = lambda: torch.cuda.Event(enable_timing=True)
    pairs = []
    for _ in range(max(args.steps, 5)):
        e1, e2 = mk(), mk()
        e1.record(stream)
        w.run(q, kv, out=o)
        e2.record(stream)
        pairs.append((e1, e2))
    torch.cuda.synchronize()
    if w.device_status():
        raise RuntimeError(f"tree attention raised device status {w.device_status()}")
    return sum(e1.elapsed_time(e2) for e1, e2 in pairs) / len(pairs)


def _bench_verify_n64(args, dev, table, stream):
    """Tree conv + GDN verify of one layer at the plugin's default tree size,
    64 nodes (fc1_fused.py:4, FC1_TREE_N), on the bench's batch and layer
    shape: the 33-64-node tensor-core verifier with its tree conv fused in
    (one launch per layer).  Mean CUDA-event time per layer over
    two alternating layers (states 128 MiB per layer: no L2 reuse)."""
    import torch
    from dforktree_b200 import workload as WL
    from dforktree_b200.cycle import CycleConfig, DraftTreeCycle
    cfg = CycleConfig(B=args.batch, layers=2, N=64)
    cyc = DraftTreeCycle(cfg, table, dev, seed=7)
    inp = WL.cycle_inputs(cfg, dev, seed=99)
    cyc.build(inp["logits"], inp["root"], inp["pre1"])
    for _ in range(max(args.warmup, 3)):
        for l in range(2):
            cyc.verify_layer(l, inp["x"][l], inp["a"][l], inp["b"][l])
    mk = lambda: torch.cuda.Event(enable_timing=True)
    pairs = []
    for _ in range(max(args.steps, 5)):
        for l in range(2):
            e1, e2 = mk(), mk()
            e1.record(stream)
            cyc.verify_layer(l, inp["x"][l], inp["a"][l], inp["b"][l])
            e2.record(stream)
            pairs.append((e1, e2))
    torch.cuda.synchronize()
    if int(cyc.status.item()):
        raise RuntimeError(f"N=64 verify raised device status {int(cyc.status.item())}")
    depth = float(cyc.tree["depth"].max(1).values.float().mean())
    ms = sum(e1.elapsed_time(e2) for e1, e2 in pairs) / len(pairs)
    del cyc, inp
    torch.cuda.empty_cache()
    return ms, depth


def run_profile_attention(args):
    """--profile-attn: W + K attention layers alone at the bench's shape (for ncu); prints nothing."""
    import torch
    from dforktree_b200 import build as B
    from dforktree_b200 import kernels as K
    B.build()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    Bt = args.batch
    par = torch.zeros(Bt, N, dtype=torch.int64, device=dev)
    par[:, 1:] = torch.randint(0, 1 << 30, (Bt, N - 1), device=dev, generator=g) % torch.arange(1, N, device=dev)
    anc = K.tree_struct(par)[0]
    w, q, kv, o = _attention_inputs(dev, Bt, anc, g)
    for _ in range(args.warmup + args.steps):
        w.run(q, kv, out=o)
    torch.cuda.synchronize()
    if w.device_status():
        raise RuntimeError(f"tree attention raised device status {w.device_status()}")


def run_profile_stage(args):
    """--profile-n64 / --profile-pmi ORDER: W + K launches of one stage alone at
    the bench's batch (for ncu); prints nothing.  n64: tree conv + verify of the
    plugin's default 64-node tree on two alternating layers; pmi: the dense
    PMI tensor of that n-gram order over the bench's scored logits, with a
    table that also carries 4M quadgram rows."""
    import torch
    from dforktree_b200 import build as B
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    from dforktree_b200 import workload as WL
    from dforktree_b200.cycle import CycleConfig, DraftTreeCycle
    from dforktree_b200.ngram_gpu import load_npz_arrays
    B.build()
    dev = torch.device("cuda", 0)
    quad = 4_000_000 if args.profile_pmi else 0
    table = K.Table(load_npz_arrays(synth.make_ngram_table(V, 2_000_000, 8_000_000, seed=0, n_quad=quad)),
                    beta3=60.0, device=dev)
    if args.profile_n64:
        cfg = CycleConfig(B=args.batch, layers=2, N=64)
        cyc = DraftTreeCycle(cfg, table, dev, seed=7)
        inp = WL.cycle_inputs(cfg, dev, seed=99)
        cyc.build(inp["logits"], inp["root"], inp["pre1"])
        for _ in range(args.warmup + args.steps):
            for l in range(2):
                cyc.verify_layer(l, inp["x"][l], inp["a"][l], inp["b"][l])
        torch.cuda.synchronize()
        status = int(cyc.status.item())
    else:
        cfg = CycleConfig(B=args.batch, layers=1)
        inp = WL.cycle_inputs(cfg, dev, seed=1234)
        _, ids, _ = K.score(inp["logits"])
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(args.warmup + args.steps):
            K.pmi_dense(table, ids, inp["root"], inp["pre1"], status=st, order=args.profile_pmi)
        torch.cuda.synchronize()
        status = int(st.item())
    if status:
        raise RuntimeError(f"profiled stage raised device status {status}")


def _traffic():
    """DRAM bytes per launch of the bench kernels from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ----------------------------------------------------------- reference -----
def _config(Bt, layers, world):
    return {"workload": WORKLOAD, "batch_per_gpu": Bt, "S": S, "V": V, "N": N, "M": M, "layers": layers,
            "Hk": HK, "Hv": HV, "D": D, "parallelism": f"request-sharded x{world}",
            "l2": "inputs larger than L2 (logits 1.5 GB, states 3 GiB per GPU); no flush"}


def run_reference(args):
    """The reference arm: whole cycles on the host cores (CpuCycle), W warm-up
    + K timed steps, plus the reference's own Triton / torch GPU path on GPU 0
    (a child process, so that a failure there leaves this line intact)."""
    workers = max(1, min(os.cpu_count() or 1, 64))
    cpu = CpuCycle(workers, args.batch, args.layers)
    times = []
    try:
        for step in range(args.warmup + args.steps):
            t = cpu.cycle()
            if step >= args.warmup:
                times.append(t)
        sample, kind = cpu.describe(), cpu.kind
    finally:
        cpu.close()
    total = sum(times)
    v = len(times) / total
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "cycles/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": _config(args.batch, args.layers, args.gpus),
            "cpu_baseline": {"value": v, "unit": "cycles/s", "cores": workers, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "cycles/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_reference_gpu:
        line["reference_gpu"] = _reference_gpu_child(args)
    return line


def _reference_gpu_child(args):
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference-gpu", "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--batch", str(args.batch), "--layers", str(args.layers)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE")}
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=1500, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference GPU path did not finish within 1500 s"}
    for ln in reversed(r.stdout.strip().splitlines()):
        if ln.startswith("{"):
            return json.loads(ln)
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"reference GPU path exited {r.returncode}: {tail[0][:300]}"}


def run_reference_gpu(args):
    """The reference's own GPU path for the same cycle on GPU 0, request by
    request as the plugin runs it (it asserts one request per verify,
    fc1_branch64.py:13): fc1_builder.Builder (torch, CUDA-graph replay), per GDN
    layer the conv hook's Triton kernel (fc1_conv.py:8-27, 35-44) and
    tree_kernels.tree_gdn_split (tree_kernels.py:193-208) with the hook's
    arguments (fc1_fused.py:59-75), greedy acceptance along the same target
    path (torch ops on the device), then fc1_fused.snapshots (fc1_fused.py:27-49,
    82) and the copy of the accepted snapshot / conv window into the request's
    slot that SGLang's commit then makes.  Same seeded inputs as our rank 0.
    Device time over K cycles (CUDA events), W warm-up cycles first."""
    ref = _ref_dir()
    if ref is None:
        return {"unavailable": "reference sources not installed under baseline/_ref"}
    import numpy as np
    import torch

    from dforktree_b200 import synth
    from dforktree_b200 import workload as WL
    from dforktree_b200.cycle import CycleConfig
    from oracle import reference_shim as RS

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    tdir = tempfile.mkdtemp(prefix="dft_ref_")
    npz = os.path.join(tdir, "table.npz")
    np.savez(npz, **synth.make_ngram_table(V, 2_000_000, 8_000_000, seed=0))
    os.environ["FC1_TREE_N"] = str(N)
    os.environ["FC1_NGRAM_PATH"] = npz
    os.environ.pop("FC1_CHAIN_FIRST", None)
    mods = RS.load_reference(ref, kernels=True)
    RS.patch_path_fn(mods)
    import triton
    TK, FF, FC = mods["tree_kernels"], mods["fc1_fused"], mods["fc1_conv"]
    cfg = CycleConfig(B=args.batch, layers=args.layers)
    Ls, Bt, C = cfg.layers, cfg.B, cfg.C
    inp = WL.cycle_inputs(cfg, dev, seed=1234)
    logits, root, pre1, x, a, b = (inp[k] for k in ("logits", "root", "pre1", "x", "a", "b"))
    acc_len = inp["acc_len"]
    builder = mods["fc1_builder"].Builder(logits[0])           # captures its CUDA graph (fc1_builder.py:20-23)
    os.unlink(npz)
    os.rmdir(tdir)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    conv_w = (torch.randn(Ls, C, 4, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    A_log = (torch.randn(Ls, HV, device=dev, generator=g) * 0.5).float()
    neg = -A_log.exp()
    dt_bias = (torch.randn(Ls, HV, device=dev, generator=g) * 0.5).float()
    conv_state = torch.randn(Ls, Bt, C, 3, device=dev, generator=g).to(torch.bfloat16)
    pool = torch.randn(Ls, Bt, HV, D, D, device=dev, generator=g) * 0.02      # [L, slots, H, V, K] like SGLang's
    keys = torch.empty(Ls, HV, N, D, device=dev)                               # Context (fc1_fused.py:12-20)
    values = torch.empty_like(keys)
    gains = torch.empty(Ls, HV, N, device=dev)
    anc_buf = torch.eye(N, device=dev)
    cidx_buf = torch.empty(N, 4, dtype=torch.int32, device=dev)
    iw = torch.empty(Ls, 1, N, C, 3, dtype=torch.bfloat16, device=dev)        # intermediate conv window, one slot
    inter = torch.empty(Ls, 1, N, HV, D, D, device=dev)                         # intermediate_ssm, one slot
    slots32 = torch.arange(Bt, dtype=torch.int32, device=dev)
    slots64 = slots32.long()
    zero = torch.zeros(1, dtype=torch.int64, device=dev)
    pos = torch.arange(LAYERS, device=dev)

    def request(r):
        tokens, depth, parent, anc, nxt, sib = builder(logits[r], root[r:r + 1], pre1[r:r + 1])
        anc_buf.copy_(anc)                                                # fc1_branch64.py:28-30
        cidx_buf.copy_(builder.cidx)
        for l in range(Ls):
            xv = x[l, r].t().unsqueeze(0)                                # [1, C, N] channels-first
            y = torch.empty(1, N, C, dtype=x.dtype, device=dev)
            cs = conv_state[l]
            FC.conv[(N, triton.cdiv(C, 256))](cs, xv, conv_w[l], xv, cidx_buf, slots64[r:r + 1], zero, iw[l], y, C,
                                              *cs.stride(), xv.stride(1), xv.stride(2), *iw[l].stride(),
                                              BIAS=False, BC=256, num_warps=4)
            TK.tree_gdn_split(y[0], a[l, r], b[l, r], A_log[l], dt_bias[l], pool[l][0].transpose(-1, -2), anc_buf,
                              HK, HV, D, D, aux=(keys[l], values[l], gains[l]), neg_exp_A=neg[l],
                              state_indices=slots32[r:r + 1], state_slot_stride=pool[l].stride(0))
        # greedy acceptance along the target path (the deepest node's), on the device
        d = builder.depth
        on_path = anc_buf[d.argmax()] > 0.5
        order = torch.where(on_path, d, N + 1).argsort()
        n_acc = torch.minimum(acc_len[r], on_path.sum())
        accept_index = torch.where(pos < n_acc, order[:LAYERS], -1)[None]
        last = order.gather(0, (n_acc - 1).view(1))
        ends = torch.cat((last, torch.full_like(last, -1)))
        FF.snapshots[(Ls * HV, 4, 8)](pool, keys, values, gains, anc_buf, accept_index, ends, slots64[r:r + 1], zero,
                                      inter, N, accept_index.shape[1], *pool.stride(), *inter.stride(), num_warps=4)
        pool[:, r].copy_(inter[:, 0].index_select(1, last).squeeze(1))
        conv_state[:, r].copy_(iw[:, 0].index_select(1, last).squeeze(1))

    def cycle():
        for r in range(Bt):
            request(r)

    for _ in range(max(args.warmup, 1)):
        cycle()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        t0.record(stream)
        for _ in range(args.steps):
            cycle()
        t1.record(stream)
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    return {"impl": "reference-gpu", "value": args.steps / (ms / 1e3), "unit": "cycles/s",
            "ms_per_step": ms / args.steps, "steps": args.steps, "warmup": args.warmup,
            "path": "reference Triton/torch GPU code from its installed sources, one request at a time",
            "clocks": clk.summary()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="reference arm: skip the reference's own GPU path (timed in a child process)")
    ap.add_argument("--requests", type=int, default=256,
                    help="config-4 stage: requests split over the GPUs (0 skips the stage)")
    ap.add_argument("--no-attn", dest="attn", action="store_false",
                    help="skip the tree-masked attention stage (reported under stages, outside the cycle)")
    ap.add_argument("--no-n64", dest="n64", action="store_false",
                    help="skip the 64-node verify stage (reported under stages, outside the cycle)")
    ap.add_argument("--profile", action="store_true", help="only W + K plain cycles (for ncu); prints nothing")
    ap.add_argument("--profile-attn", action="store_true",
                    help="only W + K tree-attention layers at the bench shape (for ncu); prints nothing")
    ap.add_argument("--profile-n64", action="store_true",
                    help="only W + K 64-node tree conv + verify launches at the bench's batch (for ncu); prints nothing")
    ap.add_argument("--profile-pmi", type=int, default=0, choices=(0, 2, 3, 4),
                    help="only W + K dense-PMI launches of this n-gram order at the bench's batch (for ncu)")
    args = ap.parse_args()
    if args.profile_attn:
        run_profile_attention(args)
        return
    if args.profile_n64 or args.profile_pmi:
        run_profile_stage(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    if args.impl == "reference-gpu":
        print(json.dumps(run_reference_gpu(args)), flush=True)
        return
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile:
        # before the first GPU call (spawned workers): one warm-up cycle, then one timed whole cycle
        workers = max(1, min(os.cpu_count() or 1, 64))
        cc = CpuCycle(workers, args.batch, args.layers)
        try:
            cc.cycle()
            t = cc.cycle()
            cpu = {"value": 1.0 / t, "unit": "cycles/s", "cores": workers, "kind": cc.kind,
                   "sample": "one " + cc.describe()[len("whole "):].replace("cycles:", "cycle:", 1)}
        finally:
            cc.close()
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    line = run_ours(args, rank, world, local_rank)
    if line is not None:
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
