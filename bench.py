"""Benchmark: KL forward + backward tokens/s at the LLaMA3-8B head shape, 32K context.

One step = the Q/Q (32 heads), K/K (8 heads) and V/V (8 heads) relation losses of
one layer for one sequence (n = 32768, d = 128, bf16, causal), forward and
backward through the public ``attn_kl_align`` operator, plus the scalar-loss
all-reduce over NCCL when N > 1.  Each rank owns one sequence (weak scaling,
one sequence per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line on rank 0.  ``--impl reference`` times LinearARD's
materialised CPU formulation (the numpy restatement in ``oracle/``) on the
host cores on a bounded sample and extrapolates it to the same workload.
``--impl reference-gpu`` times LinearARD's own Triton kernels (an unmodified
copy of ``kernels/attention_KL`` under ``baseline/_ref/``, not part of this
repository) on the same GPU workload through their ``attn_kl_align``, as a
context number; it prints an ``unavailable`` line when that copy is absent.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KL fwd+bwd tokens/s, LLaMA3-8B heads @32K ctx; % bf16 tensor peak"
WORKLOAD = "llama3_8b_32k"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--config", default=WORKLOAD)
    ap.add_argument("--cpu-sample-n", type=int, default=2048)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-numa", action="store_true",
                    help="leave the pinned staging buffers wherever the allocator puts them")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def backward_chunks(t: "torch.Tensor", causal: bool) -> int:
    """Chunks (one dq and one dk launch each) of the fused backward of the
    symmetric call on `t` [B, H, T, D], with lkl_backward_workspace_size bytes
    of scratch, as the library plans them (lkl_backward_plan)."""
    import ctypes

    from linearard_b200 import _lib
    from linearard_b200.attention_KL._common import problem
    prob = problem(t, t, t, t, causal, _lib.LKL_MASK_U8, None, None)
    L = _lib.lib()
    ws = L.lkl_backward_workspace_size(ctypes.byref(prob), 0)
    n = ctypes.c_int32(0)
    _lib.check(L.lkl_backward_plan(ctypes.byref(prob), 0, ws, 1, ctypes.byref(n)),
               "lkl_backward_plan")
    return n.value


# ------------------------------------------------------------------ CPU side
def cpu_sample(cfg, n: int, min_seconds: float = 10.0):
    """Time the oracle's materialised fp32 formulation (forward + backward of
    one causal rel-head at length n, d = cfg.head_dim) on all host cores and
    extrapolate to the full workload (cost grows with n^2 x rel-heads)."""
    import numpy as np

    from oracle import attn_kl_oracle as O
    rng = np.random.default_rng(0)
    d = cfg.head_dim
    s = rng.standard_normal((1, 1, n, d), dtype=np.float32)
    t = (s + 0.1 * rng.standard_normal((1, 1, n, d), dtype=np.float32)).astype(np.float32)
    times = []
    t_end = time.perf_counter() + min_seconds
    while True:
        t0 = time.perf_counter()
        loss, ls, lt = O.oracle_attn_kl_align(s, s, t, t, dtype=np.float32)
        O.oracle_grad(s, s, ls, t, t, lt, dtype=np.float32)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 2:
            break
    per_relhead = statistics.median(times)
    scale = (cfg.seq_len / n) ** 2 * cfg.rel_heads
    step_s = per_relhead * scale
    tokens_s = cfg.seq_len * cfg.batch / step_s
    return tokens_s, {"sample": f"1 causal rel-head, n={n}, d={d}, fp32 fwd+bwd, "
                                f"median of {len(times)} runs = {per_relhead:.3f} s; extrapolated "
                                f"x(n_full/n)^2 x {cfg.rel_heads} rel-heads",
                      "per_relhead_s": per_relhead}


def cpu_baseline_fit(cfg, n_small: int = 2048, n_large: int = 4096):
    """The CPU baseline at two lengths: the cost exponent fitted between them
    (the n^2 extrapolation assumes 2) and the extrapolation from the larger."""
    import math
    v_s, info_s = cpu_sample(cfg, n_small, min_seconds=6.0)
    v_l, info_l = cpu_sample(cfg, n_large, min_seconds=0.0)
    expo = math.log(info_l["per_relhead_s"] / info_s["per_relhead_s"]) / math.log(n_large / n_small)
    info_l["sample"] += (f"; also n={n_small}: {info_s['per_relhead_s']:.3f} s per rel-head "
                         f"(fitted cost exponent {expo:.2f} between n={n_small} and {n_large})")
    info_l["exponent_fit"] = expo
    info_l["per_n_tokens_s"] = {str(n_small): v_s, str(n_large): v_l}
    return v_l, info_l


def use_all_cpu_threads():
    """The CPU baseline runs on every host core, even under torchrun (which
    sets OMP_NUM_THREADS=1 for its workers)."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    return n


def cpu_threads():
    try:
        import numpy  # noqa: F401
        from threadpoolctl import threadpool_info
        return max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
    except Exception:
        return os.cpu_count()


def run_reference(args):
    """--impl reference: LinearARD's materialised CPU formulation on the host."""
    from linearard_b200.synth import CONFIGS
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    use_all_cpu_threads()
    for _ in range(args.warmup):
        cpu_sample(cfg, args.cpu_sample_n, min_seconds=0.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, info = cpu_sample(cfg, args.cpu_sample_n, min_seconds=0.0)
        vals.append(v)
    wall = time.perf_counter() - t0
    v = statistics.median(vals)
    cores = cpu_threads()
    out = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cfg.seq_len / v * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(cfg, args.gpus),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": info["sample"] + "; LinearARD's materialised formulation "
                         "(test_kernel_*.py reference_* / integration.py:102-127) restated in numpy"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "sample_wall_s": wall,
    }
    print(json.dumps(out), flush=True)


def config_block(cfg, n):
    return {"workload": cfg.name, "relations": "Q/Q x%d, K/K x%d, V/V x%d" % (
        cfg.q_heads, cfg.kv_heads, cfg.kv_heads), "seq_len": cfg.seq_len,
        "head_dim": cfg.head_dim, "batch_per_gpu": cfg.batch, "global_batch": cfg.batch * n,
        "causal": cfg.causal, "rope_theta": cfg.theta,
        "l2": "inputs >= 768 MiB per step (> 126 MB L2); no flush needed",
        "parallelism": f"dp{n} (one sequence per GPU, scalar loss all-reduced)"}


# ------------------------------------------------------------------ reference Triton kernels
def run_reference_gpu(args):
    """--impl reference-gpu: LinearARD's Triton attn_kl_align (integration.py:70-73
    -> kernel_A.py:190, kernel_B.py:249, kernel_C.py:293), unmodified, from
    baseline/_ref, on the same synthetic relations, timed like our arm."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    rank = int(os.environ.get("RANK", "0"))
    if not os.path.exists(os.path.join(ref_root, "kernels", "attention_KL", "integration.py")):
        if rank == 0:
            print(json.dumps({"impl": "reference-gpu", "unavailable":
                              "no copy of LinearARD's kernels/attention_KL under baseline/_ref"}))
        return
    import torch
    sys.path.insert(0, ref_root)
    from kernels.attention_KL.integration import attn_kl_align as ref_align

    from linearard_b200.synth import CONFIGS, make_relations
    if rank != 0:
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    rels = make_relations(cfg, device=dev, seed=0)
    students = {r: st.requires_grad_(True) for r, (st, _) in rels.items()}

    def step():
        total = None
        for r in cfg.relations:
            l = ref_align(students[r], students[r], rels[r][1], rels[r][1], None, cfg.causal)
            total = l if total is None else total + l
        total.backward()
        for t in students.values():
            t.grad = None
        return total.detach()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(args.steps):
            loss = step()
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    value = cfg.seq_len * cfg.batch / (ms / 1e3)
    print(json.dumps({
        "impl": "reference-gpu", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": config_block(cfg, 1), "step_tflops": cfg.algorithmic_flops() / (ms / 1e3) / 1e12,
        "clocks": clk.summary(), "loss": float(loss),
        "what": "LinearARD's Triton kernels (unmodified copy under baseline/_ref), same step"}),
        flush=True)


def gpu_local_cpus(dev):
    """CPUs of the NUMA node that the GPU's PCIe device reports (sysfs
    local_cpulist), or None when that cannot be read."""
    try:
        import torch
        pr = torch.cuda.get_device_properties(dev)
        bus = "%04x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            if "-" in part:
                a, b = part.split("-")
                cpus.update(range(int(a), int(b) + 1))
            elif part:
                cpus.add(int(part))
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:  # noqa: BLE001 -- no sysfs entry / no PCI info: leave placement alone
        return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ GPU side
def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.impl == "reference-gpu":
        run_reference_gpu(args)
        return

    import torch
    import torch.distributed as dist

    from linearard_b200 import _lib, attn_kl_align
    from linearard_b200.synth import CONFIGS, make_relations

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    cfg = CONFIGS[args.config]
    L = _lib.lib()

    # inputs for this rank's sequence (seeded by rank: no scatter needed)
    rels = make_relations(cfg, device=dev, seed=1000 * rank)
    students = {r: st.requires_grad_(True) for r, (st, _) in rels.items()}
    teachers = {r: te for r, (_, te) in rels.items()}

    def step(S, Tt, marks=None):
        """marks: three CUDA events recorded at the start, after the forward
        calls and at the end of the step (the live forward / backward split)."""
        if marks:
            marks[0].record()
        total = None
        for r in cfg.relations:
            l = attn_kl_align(S[r], S[r], Tt[r], Tt[r], None, cfg.causal)
            total = l if total is None else total + l
        if marks:
            marks[1].record()
        total.backward()
        if marks:
            marks[2].record()
        if world > 1:
            red = total.detach().clone()
            dist.all_reduce(red)
            return red
        return total.detach()

    def zero_grads(S):
        for t in S.values():
            t.grad = None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timing
    for _ in range(args.warmup):
        zero_grads(students)
        step(students, teachers)
    assert L.lkl_last_path() == 1, "tensor-core kernels not selected"
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        marks = [[torch.cuda.Event(enable_timing=True) for _ in range(3)]
                 for _ in range(args.steps)]
        ev0.record()
        for k in range(args.steps):
            zero_grads(students)
            loss = step(students, teachers, marks[k])
        ev1.record()
        barrier()
    ms = ev0.elapsed_time(ev1)
    t_max = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    ms_step = ms / args.steps
    tokens = cfg.seq_len * cfg.batch * world * args.steps
    value = tokens / (ms / 1e3)
    st = L.lkl_device_status()
    assert st == 0, f"device status {st}"
    # per relation: forward kernel + loss reduction; backward: lse pre-pass, then
    # a dq and a dk launch per chunk of the D-tile buffer
    launches_per_step = sum(3 + 2 * backward_chunks(students[r].detach(), cfg.causal)
                            for r in cfg.relations)

    # ---- forward / backward split of the timed steps (events inside the
    # timed region, on the stream every launch of the step goes to)
    fwd_ms = [m[0].elapsed_time(m[1]) for m in marks]
    bwd_ms = [m[1].elapsed_time(m[2]) for m in marks]
    n, d = cfg.seq_len, cfg.head_dim
    heads = sum(cfg.heads(r) for r in cfg.relations) * cfg.batch
    flops_fwd = 2.0 * n * n * d * heads   # 2 causal n x n x d contractions per rel-head
    flops_bwd = 4.0 * n * n * d * heads   # 4 causal contractions per rel-head
    peaks, peak_kind = load_peaks()
    peak = peaks["bf16_tflops"]
    peak_sus = peaks.get("bf16_tflops_sustained", peak)
    t_fwd, t_bwd = sum(fwd_ms) / len(fwd_ms) / 1e3, sum(bwd_ms) / len(bwd_ms) / 1e3
    dom = "bwd" if t_bwd >= t_fwd else "fwd"
    dom_flops, dom_t = (flops_bwd, t_bwd) if dom == "bwd" else (flops_fwd, t_fwd)
    achieved = dom_flops / dom_t / 1e12
    step_tflops = cfg.algorithmic_flops() / (ms_step / 1e3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("backward_kernels" if dom == "bwd" else "sm100_forward_kernel")

    # ---- end to end from pinned host buffers through the public API
    e2e = None
    if not args.no_e2e:
        # Each step's inputs come from pinned host memory through the public
        # API, as a training loop with a prefetching loader runs it: two sets
        # of device input buffers; while step k computes on set k % 2, a copy
        # stream fills set (k + 1) % 2 with step k + 1's inputs (after step
        # k - 1, the last user of that set, is done).  Every step carries one
        # full host->device copy of its inputs and one device->host read of its
        # loss (into pinned memory; the host reads step k - 1's loss during
        # step k, so the GPU never waits for the host).
        numa = None if args.no_numa else gpu_local_cpus(dev)
        saved_affinity = None
        if numa:
            # pinned staging pages are placed on the NUMA node of this GPU's
            # PCIe root (first touch by a thread running there), so the copy
            # engines of N GPUs do not all read across the socket link
            saved_affinity = os.sched_getaffinity(0)
            os.sched_setaffinity(0, numa)
        host = [(students[r].detach().cpu().pin_memory(), teachers[r].cpu().pin_memory())
                for r in cfg.relations]
        loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
        if saved_affinity is not None:
            os.sched_setaffinity(0, saved_affinity)
        bufs = [[(torch.empty_like(hs, device=dev), torch.empty_like(ht, device=dev))
                 for hs, ht in host] for _ in range(2)]
        h2d = sum(x.numel() * x.element_size() for pair in host for x in pair)
        copy_stream = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        loss_ready = [torch.cuda.Event() for _ in range(2)]
        state = {"k": 0, "last": None}

        def prefetch(k):
            """Copies of step k's inputs into buffer set k % 2 (copy stream)."""
            with torch.cuda.stream(copy_stream):
                if k >= 2:
                    copy_stream.wait_event(done[k % 2])   # step k - 2 is done with the set
                for (hs, ht), (ds, dt) in zip(host, bufs[k % 2]):
                    ds.copy_(hs, non_blocking=True)
                    dt.copy_(ht, non_blocking=True)
                copied[k % 2].record(copy_stream)

        def e2e_step():
            k = state["k"]
            cur = torch.cuda.current_stream(dev)
            if k == 0:
                prefetch(0)
            prefetch(k + 1)                  # runs under this step's compute
            cur.wait_event(copied[k % 2])
            total = None
            for ds, dt in bufs[k % 2]:
                s_leaf = ds.detach().requires_grad_(True)
                l = attn_kl_align(s_leaf, s_leaf, dt, dt, None, cfg.causal)
                total = l if total is None else total + l
            total.backward()
            if world > 1:
                red = total.detach().clone()
                dist.all_reduce(red)
                total = red
            loss_host[k % 2].copy_(total.detach(), non_blocking=True)   # device -> host
            loss_ready[k % 2].record(cur)
            done[k % 2].record(cur)
            if k > 0:                        # the host reads the previous step's loss
                loss_ready[(k - 1) % 2].synchronize()
                state["last"] = float(loss_host[(k - 1) % 2])
            state["k"] = k + 1

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        for _ in range(args.steps):
            e2e_step()
        torch.cuda.current_stream(dev).wait_stream(copy_stream)   # the last prefetch too
        k1.record()
        barrier()
        e_ms = torch.tensor([k0.elapsed_time(k1)], device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        # the host path alone: the same copies, every rank at once, no compute
        # (the ceiling the overlapped step can approach)
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(copy_stream)
        with torch.cuda.stream(copy_stream):
            for _ in range(args.steps):
                for (hs, ht), (ds, dt) in zip(host, bufs[0]):
                    ds.copy_(hs, non_blocking=True)
                    dt.copy_(ht, non_blocking=True)
        c1.record(copy_stream)
        barrier()
        c_ms = torch.tensor([c0.elapsed_time(c1) / args.steps], device=dev)
        if world > 1:
            dist.all_reduce(c_ms, op=dist.ReduceOp.MAX)
        e_step = float(e_ms.item()) / args.steps
        copy_ms = float(c_ms.item())
        e2e = {"value": tokens / (float(e_ms.item()) / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4,
               "ms_per_step": e_step,
               "h2d_copy_only_ms_per_step": copy_ms,
               "h2d_gbs_per_rank_copy_only": h2d / (copy_ms / 1e3) / 1e9,
               "exposed_ms_per_step": e_step - ms_step,
               "bound": "host->device copies" if copy_ms >= ms_step else "device compute",
               "staging_numa_local": bool(numa),
               "input_pipeline": "two device input sets: step k+1's copies run under step k; "
                                 "loss read one step behind into pinned memory"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        use_all_cpu_threads()
        v, info = cpu_baseline_fit(cfg)
        cpu = {"value": v, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": info["sample"], "exponent_fit": info["exponent_fit"],
               "tokens_s_by_sample_n": info["per_n_tokens_s"]}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded Gaussian + RoPE theta=5e5, student "
                                     "positions/8; BASELINE configs[2])",
            "config": config_block(cfg, world),
            "tensor_peak_frac": step_tflops / peak,
            "tensor_peak_frac_sustained": step_tflops / peak_sus,
            "step_tflops": step_tflops,
            "roofline": {"bound": "tensor",
                         "kernel": ("backward of the step: sm100_dq_kernel + sm100_dk_kernel launches "
                                    "(with the LSE pre-pass and the autograd cast)"
                                    if dom == "bwd" else "sm100_forward_kernel"),
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} bf16_tflops (burst)",
                         "peak_sustained": peak_sus, "frac_sustained": achieved / peak_sus,
                         "fwd_ms": t_fwd * 1e3, "bwd_ms": t_bwd * 1e3,
                         "split": "forward calls / backward of the timed steps (CUDA events)",
                         "fwd_tflops": flops_fwd / t_fwd / 1e12,
                         "bwd_tflops": flops_bwd / t_bwd / 1e12},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
            "loss": float(loss.item()),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
