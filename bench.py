"""Benchmark of the fused per-layer path (one JSON line on rank 0).

Metric: fused-layer tokens/s/GPU at T=512, and HBM GB/s as a
fraction of 8 TB/s, on 1/2/4/8 B200.

A "step" is one pass of the hot path over one 512-token prefill chunk per GPU
(the engine's chunk size, src/ds3.h:82), through the ds3_cuda C-ABI:
  1. embed_rms_norm        Q4_K token_embd gather + dequant + attn_norm
  2. qk_norm_rope          per-head Q/K RMSNorm + NEOX RoPE (32 Q / 4 KV heads)
  3. add_rms_norm          residual add + ffn_norm
  4. router_softmax_topk   softmax over 128 experts, top-8, renorm
  5. swiglu                silu(gate)*up * routing weight, 4096 x 768
  6. moe_combine_residual  weighted sum of 8 expert rows + residual
The projections between these ops (QKV/O, router logits, expert matmuls) are
out of scope; their outputs are seeded synthetic tensors of the right shapes.
Scaling is weak: every GPU runs its own 512-token chunk, with no collective.

value   : whole-job tokens/s over all N GPUs (the bench contract's aggregate;
          tokens/s/GPU, the metric's own unit, is tokens_per_s_per_gpu =
          value / N), inputs resident in HBM (K graph replays, CUDA events on
          the module stream, barrier + synchronize both sides, max over ranks).
          Inputs rotate over several sets larger than L2 together.
parity  : one step of every rank compared with the oracle before timing; under
          torchrun the step outputs of all ranks are all-gathered with NCCL and
          rank 0 checks every row of the whole job.
e2e     : same step through the C-ABI from pinned host buffers, host->device
          copies of every input and device->host read of the outputs timed;
          its roofline is the pinned host<->device copy rate measured in the
          same run (all ranks copying at once).
roofline: the kernel with the largest share of the step, algorithmic bytes per
          launch / its average CUDA-event duration, against the measured HBM
          copy peak.
--impl reference: the reference's own CPU kernels (oracle/_ref, the unmodified
          src/ds3_reference.c) on the same workload, all host threads, rank 0,
          whole 512-token steps for at least 5 s; the single-thread rate (as
          the reference runs) is reported beside it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from qw3_b200 import inputs as I  # noqa: E402

METRIC = "fused-layer tokens/s/GPU at T=512 and HBM GB/s as % of 8 TB/s, 1/2/4/8 B200"
T = 512
H = I.N_EMBD
NQ, NK, HD = I.N_HEAD, I.N_HEAD_KV, I.HEAD_DIM
E, K = I.N_EXPERT, I.N_EXPERT_USED
FF = I.N_FF_EXP
V = I.N_VOCAB
Q4K_ROW = H // 256 * 144
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0

# Algorithmic bytes per launch (per 512-token chunk): what each op must read
# and write at least once. Shared parameters (gammas, frequency table) are
# not counted; only the gathered embedding rows are.
ALGO_BYTES = {
    "embed_rms_norm": T * (Q4K_ROW + 4 + 4 * H + 4 * H),
    "qk_norm_rope": T * (2 * 4 * (NQ + NK) * HD + 4),
    "add_rms_norm": T * 4 * H * 4,
    "router_softmax_topk": T * (4 * E + 4 * K + 4 * K),
    "swiglu": T * K * (3 * 4 * FF + 4),
    "moe_combine_residual": T * (K * 4 * H + 4 * H + 4 * K + 4 * H),
}
OPS = list(ALGO_BYTES)
STEP_BYTES = sum(ALGO_BYTES.values())

# DRAM traffic per launch measured with ncu (dram__bytes_read.sum +
# dram__bytes_write.sum, --clock-control none), one capture per kernel on
# this workload. Reads equal
# the algorithmic input bytes; the outputs of one T=512 launch are still in
# L2 when it ends, so no write traffic is attributed to the launch itself.
NCU_TRAFFIC = {
    "embed_rms_norm": 638976,
    "qk_norm_rope": 9458944,
    "add_rms_norm": 8412416,
    "router_softmax_topk": 271360,
    "swiglu": 25196544,
    "moe_combine_residual": 37777408,
}

N_SETS = 4  # input sets rotated between steps (each ~73 MB; together > 126 MB L2)

CONFIG = {
    "workload": "fused_layer_T512",
    "tokens_per_gpu": T,
    "ops": OPS,
    "table": "Q4_K token_embd 151936x2048 (175 MB, device-resident)",
    "model_dims": "Qwen3-30B-A3B: n_embd 2048, 32 Q / 4 KV heads x 128, 128 experts top-8, n_ff_exp 768",
    "parallelism": "row shard, one 512-token chunk per GPU, no collective",
    "l2": "inputs larger than L2: steps rotate over %d input sets of ~73 MB each (~292 MB) plus the 175 MB table"
          % N_SETS,
}


def config_line(world: int) -> dict:
    """The `config` both arms print (so the driver sees the same workload)."""
    return dict(CONFIG, global_tokens=world * T)


# --------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def make_host_set(seed: int, table_rows: int = V):
    """One step's inputs (numpy, host) for a 512-token chunk."""
    g = {}
    g["ids"] = I.token_ids(T, seed + 0, table_rows)
    g["pos"] = np.arange(T, dtype=np.int32)
    g["q"] = I.normal(seed + 1, (T, NQ, HD))
    g["k"] = I.normal(seed + 2, (T, NK, HD))
    g["attn_out"] = I.normal(seed + 3, (T, H))
    g["logits"] = I.normal(seed + 4, (T, E), 0.0, 2.0)
    g["gate"] = I.normal(seed + 5, (T * K, FF), 0.0, 1.5)
    g["up"] = I.normal(seed + 6, (T * K, FF), 0.0, 1.5)
    g["y"] = I.normal(seed + 7, (T * K, H))
    return g


def make_params():
    return {
        "attn_norm": I.gamma(H, 1101),
        "ffn_norm": I.gamma(H, 1102),
        "q_norm": I.gamma(HD, 1103),
        "k_norm": I.gamma(HD, 1104),
    }


class DevSet:
    """Device buffers for one step (inputs + outputs)."""

    IN = ["ids", "pos", "q", "k", "attn_out", "logits", "gate", "up", "y"]

    def __init__(self, ds3, host):
        self.b = {n: ds3.upload(host[n]) for n in self.IN}
        for n, nbytes in (("hidden", T * H * 4), ("xnorm", T * H * 4), ("resid", T * H * 4),
                          ("ffn_in", T * H * 4), ("idx", T * K * 4), ("scores", T * K * 4),
                          ("act", T * K * FF * 4), ("out", T * H * 4)):
            self.b[n] = ds3.empty(nbytes)

    def free(self):
        for b in self.b.values():
            b.free()


def enqueue_step(ds3, P, S, marks=None):
    """Enqueue the six ops of one step; with `marks` (list of timer slots),
    record a timer event before the first op and after every op."""
    b = S.b
    eps = I.NORM_EPS

    def mark(i):
        if marks is not None:
            ds3.timer_mark(marks[i])

    mark(0)
    rc = ds3.embed_rms_norm(P["table"], b["ids"], P["attn_norm"], b["hidden"], b["xnorm"], T, H, V,
                            ds3.TYPE_Q4_K, Q4K_ROW, eps)
    mark(1)
    rc |= ds3.qk_norm_rope(b["q"], b["k"], P["q_norm"], P["k_norm"], b["pos"], T, NQ, NK, HD, I.ROPE_THETA, eps)
    mark(2)
    rc |= ds3.add_rms_norm(b["attn_out"], b["hidden"], P["ffn_norm"], b["resid"], b["ffn_in"], H, T, eps)
    mark(3)
    rc |= ds3.router_softmax_topk(b["logits"], None, b["idx"], b["scores"], T, E, K, True)
    mark(4)
    rc |= ds3.swiglu(b["gate"], b["up"], b["scores"], b["act"], T * K, FF)
    mark(5)
    rc |= ds3.moe_combine_residual(b["y"], None, b["scores"], b["resid"], b["out"], T, K, H)
    mark(6)
    if rc != 0:
        raise RuntimeError("enqueue failed: " + ds3.last_error())


# ------------------------------------------------------------------ NVML
def nvml_handle(device_index: int):
    """NVML handle of CUDA device `device_index` of this process, matched by
    PCI address (NVML numbers devices physically, CUDA after
    CUDA_VISIBLE_DEVICES), or None."""
    try:
        import pynvml
        import torch

        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(device_index)
        bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        try:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.upper())
    except Exception:
        return None


def bind_to_gpu_cpus(device_index: int):
    """Run this rank on the host cores NVML lists as local to its GPU, so its
    pinned host buffers are allocated (first touch) on the GPU's own NUMA node
    and its copies do not cross the socket link. Returns the core count, or
    None when NVML cannot tell (nothing is changed then)."""
    h = nvml_handle(device_index)
    if h is None:
        return None
    try:
        import pynvml

        n = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:
        return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.0005):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = nvml_handle(device_index)
            if self.h is None:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report nothing rather than guess
            self.nv = None

    def _sample(self):
        self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
        try:
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()
            self._sample()  # the end of the timed region, however short it was

    def summary(self):
        if not self.nv or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            v = float(json.loads(p.read_text())["hbm_gbs"])
            return v, "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------ CPU reference
def cpu_oracle():
    import oracle

    oracle.build() if not oracle.PORT_LIB.exists() else None
    ref = oracle.reference()
    if ref is not None:
        return ref, "reference"
    return oracle.port(), "port"


def cpu_step(O, table, params, g, n_tok, threads):
    """The same six ops on the host CPU for the first n_tok tokens of set g."""
    eps = I.NORM_EPS
    ids = g["ids"][:n_tok]
    _, hid, _ = O.embed_rms_norm(table, 12, Q4K_ROW, V, ids, H, params["attn_norm"], eps, threads)
    O.qk_norm_rope(g["q"][:n_tok], g["k"][:n_tok], params["q_norm"], params["k_norm"], g["pos"][:n_tok],
                   I.ROPE_THETA, eps, threads)
    s, _ = O.add_rms_norm(g["attn_out"][:n_tok], hid, params["ffn_norm"], eps, threads)
    _, _, sc = O.router(g["logits"][:n_tok], K, True, threads)
    O.swiglu(g["gate"][: n_tok * K], g["up"][: n_tok * K], sc.reshape(-1), threads)
    O.combine(g["y"][: n_tok * K], sc, s, None, threads)


def time_cpu(O, table, params, g, threads, budget_s=10.0, max_steps=None):
    """Tokens/s of the CPU path on a bounded sample: whole 512-token steps
    until `budget_s` is spent (at least one); sub-chunks if one step is
    longer than the budget."""
    for _ in range(2):  # warm caches, page in the table rows, start the thread pool
        cpu_step(O, table, params, g, T, threads)
    t0 = time.perf_counter()
    cpu_step(O, table, params, g, T, threads)
    probe = time.perf_counter() - t0
    n_tok = T if probe <= budget_s else max(8, int(T * budget_s / probe / 4))
    steps, tok = 0, 0
    t0 = time.perf_counter()
    while True:
        cpu_step(O, table, params, g, n_tok, threads)
        steps += 1
        tok += n_tok
        el = time.perf_counter() - t0
        if el >= budget_s or (max_steps and steps >= max_steps):
            break
    return tok / el, {"tokens": tok, "steps": steps, "tokens_per_step": n_tok, "seconds": round(el, 3)}


def cpu_baseline(O, kind, table, params, g, budget_all=10.0, budget_one=5.0):
    """The reference's CPU path on this host: all cores (the reported value)
    and one thread (as the reference itself runs, src/ds3_reference.h:5)."""
    thr = cpu_cores()
    v_all, s_all = time_cpu(O, table, params, g, thr, budget_all)
    v_one, s_one = time_cpu(O, table, params, g, 1, budget_one)

    def sample(sm, n):
        return (f"{sm['steps']} steps x {sm['tokens_per_step']} tokens of the same workload, {n} thread(s), "
                f"{sm['seconds']} s")

    return {"value": round(v_all, 2), "unit": "tokens/s", "cores": thr, "kind": kind, "sample": sample(s_all, thr),
            "threads_all": {"value": round(v_all, 2), "threads": thr, "sample": sample(s_all, thr)},
            "threads_1": {"value": round(v_one, 2), "threads": 1, "sample": sample(s_one, 1)}}


def run_reference(args, rank, world):
    """The reference's own CPU kernels on the GPU arm's workload: each of the
    K timed steps runs `reps` whole 512-token passes, with `reps` sized so the
    timed region lasts at least 5 s (and the whole run a few minutes)."""
    if rank != 0:
        return 0
    O, kind = cpu_oracle()
    threads = cpu_cores()
    table = I.q4k_table(V, H, 1)
    params = make_params()
    g = make_host_set(seed=2000)
    for _ in range(2):
        cpu_step(O, table, params, g, T, threads)
    full = 1e9
    for _ in range(3):  # the fastest of three whole passes sizes the sample
        t0 = time.perf_counter()
        cpu_step(O, table, params, g, T, threads)
        full = min(full, time.perf_counter() - t0)
    reps = max(1, int(np.ceil(5.5 / (max(args.steps, 1) * full))))
    if full * reps * (args.steps + args.warmup) > 150.0:  # keep the run within a few minutes
        reps = max(1, int(150.0 / (full * (args.steps + args.warmup))))
    for _ in range(args.warmup):
        cpu_step(O, table, params, g, T, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(reps):
            cpu_step(O, table, params, g, T, threads)
    el = time.perf_counter() - t0
    value = T * reps * args.steps / el
    sample = f"{args.steps} steps x {reps} whole 512-token passes, {threads} threads, {el:.2f} s"
    v_one, s_one = time_cpu(O, table, params, g, 1, 5.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * el / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; no dataset or weights exist for this path)", "config": config_line(world),
        "value_is": "tokens/s of the reference's CPU kernels on rank 0's host (all threads)",
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": sample,
                         "threads_all": {"value": round(value, 2), "threads": threads, "sample": sample},
                         "threads_1": {"value": round(v_one, 2), "threads": 1,
                                       "sample": f"{s_one['steps']} steps x {s_one['tokens_per_step']} tokens, "
                                                 f"1 thread, {s_one['seconds']} s"}},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "hbm_gbs_per_gpu": None,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sets", type=int, default=N_SETS, help="input sets rotated to defeat L2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-config kernel lines")
    ap.add_argument("--shard-of", type=int, default=0, metavar="N",
                    help="with --only-configs: run the C4/C5 row shard one GPU of N would hold")
    ap.add_argument("--only-configs", action="store_true",
                    help="run only the per-config kernels (a short command for ncu captures)")
    ap.add_argument("--profile", action="store_true", help="short run for ncu: no e2e, baseline or configs")
    ap.add_argument("--rope-f16", type=int, default=0, metavar="T",
                    help="time only QK-norm+RoPE with fp16 storage on T tokens (a small case for ncu)")
    ap.add_argument("--router-proj", type=int, default=0, metavar="T",
                    help="time only the router projection + top-8 on T tokens (a small case for ncu)")
    ap.add_argument("--decode-ffn", type=int, default=0, metavar="T",
                    help="time only the fused add + ffn_norm + router projection + top-8 on T tokens")
    ap.add_argument("--expert-lists", type=int, default=0, metavar="T",
                    help="time only the device per-expert token lists for T tokens (a small case for ncu)")
    ap.add_argument("--cycle-graph", type=int, default=1,
                    help="capture one graph of a step on every input set in turn (1) or time single-step graphs (0)")
    ap.add_argument("--pdl", type=int, default=1, help="programmatic dependent launch between ops (1/0)")
    args = ap.parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    args.warmup = max(args.warmup, 3)
    # Only the JSON line may reach stdout: libraries (NCCL's banner, CUDA
    # messages) write to fd 1 directly, so fd 1 is pointed at stderr and the
    # line is written to a duplicate of the original stdout.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)

    def emit(obj):
        os.write(json_fd, (json.dumps(obj) + "\n").encode())

    import torch

    torch.cuda.set_device(local)
    # Under torchrun every rank copies its own step inputs from pinned host
    # memory (e2e); keep each rank on its GPU's local cores and memory.
    host_cores = bind_to_gpu_cpus(local) if world > 1 else None
    if world > 1:
        import torch.distributed as dist

        # NCCL's INIT log (communicator rank counts) goes to fd 1, which now
        # points at stderr; a caller's own NCCL_DEBUG setting is kept.
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    os.environ["DS3_CUDA_PDL"] = str(args.pdl)
    from qw3_b200 import ds3

    if ds3.set_device(local) != 0 or ds3.init() != 0:
        raise SystemExit("ds3_cuda_init failed: " + ds3.last_error())

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def all_ranks(x: float) -> list:
        if world == 1:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        parts = [torch.empty_like(t) for _ in range(world)]
        torch.distributed.all_gather(parts, t)
        return [float(p.item()) for p in parts]

    if args.rope_f16 or args.router_proj or args.expert_lists or args.decode_ffn:
        if args.rope_f16:
            line = run_rope_f16(ds3, args.rope_f16, max_over_ranks, barrier)
        elif args.decode_ffn:
            line = run_decode_ffn(ds3, args.decode_ffn, max_over_ranks, barrier)
        elif args.router_proj:
            line = run_router_proj(ds3, args.router_proj, max_over_ranks, barrier)
        else:
            line = run_expert_lists(ds3, args.expert_lists, max_over_ranks, barrier)
        if rank == 0:
            emit(line)
        return 0

    # ---- inputs: table shared by all steps, S rotating sets of activations
    table_host = I.q4k_table(V, H, 1)
    if args.only_configs:
        peak, _ = measured_peak()
        cfg = run_configs(ds3, world, rank, max_over_ranks, barrier, peak, table_host, args.shard_of)
        if rank == 0:
            emit({"configs": cfg, "shard_of": args.shard_of})
        return 0
    params_host = make_params()
    P = {"table": ds3.buffer_from_mmap(table_host)}
    for n, a in params_host.items():
        P[n] = ds3.upload(a)
    hosts = [make_host_set(seed=set_seed(s, rank)) for s in range(args.sets)]
    sets = [DevSet(ds3, h) for h in hosts]

    # ---- parity of one step (set 0 of every rank) against the oracle before
    # timing; under torchrun the outputs of all ranks are gathered with NCCL
    # and rank 0 checks the whole job.
    enqueue_step(ds3, P, sets[0])
    ds3.synchronize()
    parity = job_parity(ds3, table_host, params_host, sets[0], rank, world)
    # restore the in-place Q/K of set 0
    ds3.buffer_write(sets[0].b["q"], 0, hosts[0]["q"])
    ds3.buffer_write(sets[0].b["k"], 0, hosts[0]["k"])

    # ---- graphs: one per input set
    graphs = []
    for S in sets:
        ds3.graph_begin()
        enqueue_step(ds3, P, S)
        graphs.append(ds3.graph_end())

    # One more graph holds a step on every input set in turn, so that the
    # programmatic overlap also spans step boundaries (an engine captures a
    # whole forward pass the same way); the timed loop replays it K // S
    # times and the single-step graphs for the remainder: exactly K steps.
    cycle = None
    if args.cycle_graph and len(sets) > 1:
        ds3.graph_begin()
        for S in sets:
            enqueue_step(ds3, P, S)
        cycle = ds3.graph_end()

    def run_steps(k):
        if cycle is not None:
            for _ in range(k // len(sets)):
                ds3.graph_launch(cycle)
            for i in range(k % len(sets)):
                ds3.graph_launch(graphs[i])
        else:
            for i in range(k):
                ds3.graph_launch(graphs[i % len(graphs)])

    run_steps(args.warmup)
    ds3.synchronize()

    clocks = ClockSampler(local)
    barrier()
    ds3.synchronize()
    clocks.start()
    ds3.timer_mark(0)
    run_steps(args.steps)
    ds3.timer_mark(1)
    ds3.synchronize()
    clocks.stop()
    barrier()
    ms_rank = ds3.timer_elapsed_ms(0, 1)
    per_rank = [m / args.steps for m in all_ranks(ms_rank)]
    ms_step = max(per_rank)
    value = world * T / (ms_step * 1e-3)

    # ---- per-kernel durations: each op alone, back to back, over copies of
    # its operands that together exceed L2 (so every launch streams from HBM)
    peak, peak_kind = measured_peak()
    kernels = op_loops(ds3, P, max_over_ranks, barrier, peak)
    if not args.profile:
        stream_floor(ds3, kernels, max_over_ranks, barrier)
    tot = sum(k["avg_us"] for k in kernels.values())
    for k in kernels.values():
        k["share"] = round(k["avg_us"] / tot, 4)
    dom = max(kernels, key=lambda o: kernels[o]["avg_us"])
    d = kernels[dom]
    roofline = {"kernel": dom, "bound": "hbm", "achieved": d["gbs"], "peak": peak, "unit": "GB/s",
                "frac": round(d["gbs"] / peak, 4), "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                "traffic": NCU_TRAFFIC.get(dom), "algo_bytes_per_launch": ALGO_BYTES[dom],
                "timing": "CUDA events around back-to-back launches of this kernel alone (graph, module stream)"}

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; no dataset or weights exist for this path)",
        "config": config_line(world),
        "value_is": "whole-job tokens/s summed over all n_gpus (the bench contract); tokens/s/GPU is "
                    "tokens_per_s_per_gpu",
        "tokens_per_s_per_gpu": round(value / world, 1),
        "ms_per_step_per_rank": [round(m, 6) for m in per_rank],
        "slowest_rank": int(np.argmax(per_rank)),
        "pdl": bool(args.pdl),
        "host_cores_per_rank": host_cores,
        "process_group": ({"backend": torch.distributed.get_backend(), "world_size": torch.distributed.get_world_size()}
                          if world > 1 else None),
        "graphs": ("one graph per %d steps (a step on each input set in turn), replayed" % len(sets))
                  if cycle is not None else "one graph per step, replayed",
        "hbm_gbs_per_gpu": round(STEP_BYTES / (ms_step * 1e-3) / 1e9, 1),
        "pct_of_8tbs": round(100 * STEP_BYTES / (ms_step * 1e-3) / 1e9 / NOMINAL_HBM_GBS, 2),
        "pct_of_measured_peak": round(100 * STEP_BYTES / (ms_step * 1e-3) / 1e9 / peak, 2),
        "step_algo_bytes": STEP_BYTES,
        "roofline": roofline,
        "kernels": kernels,
        "gpu_launches": 6 * args.steps,
        "clocks": clocks.summary(),
        "parity": parity,
    }

    if not args.profile:
        line["e2e"] = run_e2e(ds3, P, sets, hosts, args.steps, world, max_over_ranks, barrier)
        if not args.no_configs:
            line["configs"] = run_configs(ds3, world, rank, max_over_ranks, barrier, peak, table_host)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            Oc, kind = cpu_oracle()
            line["cpu_baseline"] = cpu_baseline(Oc, kind, table_host, params_host, hosts[0])
    for g in graphs + ([cycle] if cycle is not None else []):
        ds3.graph_free(g)
    if rank == 0:
        emit(line)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def set_seed(s: int, rank: int) -> int:
    return 2000 + 97 * s + 10007 * rank


def set_bytes(h):
    return sum(a.nbytes for a in h.values())


def step_outputs(ds3, S):
    b = S.b
    return {"hidden": ds3.download(b["hidden"], np.float32, (T, H)),
            "xnorm": ds3.download(b["xnorm"], np.float32, (T, H)),
            "q": ds3.download(b["q"], np.float32, (T, NQ, HD)),
            "k": ds3.download(b["k"], np.float32, (T, NK, HD)),
            "resid": ds3.download(b["resid"], np.float32, (T, H)),
            "ffn_in": ds3.download(b["ffn_in"], np.float32, (T, H)),
            "idx": ds3.download(b["idx"], np.int32, (T, K)),
            "scores": ds3.download(b["scores"], np.float32, (T, K)),
            "act": ds3.download(b["act"], np.float32, (T * K, FF)),
            "out": ds3.download(b["out"], np.float32, (T, H))}


def tol_ratio(got, want, rtol=1e-5, atol=1e-6) -> float:
    """max |got - want| / (atol + rtol |want|), in row blocks: <= 1 is within
    tolerance."""
    got = got.reshape(got.shape[0], -1)
    want = want.reshape(want.shape[0], -1)
    worst = 0.0
    for a in range(0, got.shape[0], 2048):
        g = got[a:a + 2048].astype(np.float64)
        w = want[a:a + 2048].astype(np.float64)
        worst = max(worst, float(np.max(np.abs(g - w) / (atol + rtol * np.abs(w)), initial=0.0)))
    return worst


def bitexact(got, want) -> bool:
    return got.shape == want.shape and bool(np.array_equal(np.ascontiguousarray(got).view(np.uint8),
                                                           np.ascontiguousarray(want).view(np.uint8)))


def check_outputs(O, table, params, g, out, threads):
    """Compare one step's outputs with the oracle on the same inputs: exact
    where the path is exact, else the worst error as a fraction of the
    stated tolerance: 1e-5 relative, 1e-6 absolute (<= 1 passes)."""
    eps = I.NORM_EPS
    res = {}
    _, hid, xn = O.embed_rms_norm(table, 12, Q4K_ROW, V, g["ids"], H, params["attn_norm"], eps, threads)
    res["embed_bitexact"] = bitexact(out["hidden"], hid)
    res["attn_norm_tol_ratio"] = tol_ratio(out["xnorm"], xn)
    qo, ko = O.qk_norm_rope(g["q"], g["k"], params["q_norm"], params["k_norm"], g["pos"], I.ROPE_THETA, eps,
                            threads)
    res["qk_rope_tol_ratio"] = max(tol_ratio(out["q"], qo), tol_ratio(out["k"], ko))
    s, fn = O.add_rms_norm(g["attn_out"], hid, params["ffn_norm"], eps, threads)
    res["residual_bitexact"] = bitexact(out["resid"], s)
    res["ffn_norm_tol_ratio"] = tol_ratio(out["ffn_in"], fn)
    _, idx, sc = O.router(g["logits"], K, True, threads)
    res["top8_exact"] = bitexact(out["idx"], idx)
    res["scores_tol_ratio"] = tol_ratio(out["scores"], sc)
    act = O.swiglu(g["gate"], g["up"], out["scores"].reshape(-1), threads)
    res["swiglu_tol_ratio"] = tol_ratio(out["act"], act)
    o = O.combine(g["y"], out["scores"], s, None, threads)
    res["combine_bitexact"] = bitexact(out["out"], o)
    return res


def parity_ok(res: dict) -> bool:
    return all((v <= 1.0) if k.endswith("tol_ratio") else bool(v) for k, v in res.items() if k != "ok")


def job_parity(ds3, table, params, S, rank, world):
    """One step of every rank against the oracle. With N > 1 the step
    outputs are all-gathered over NCCL (shard.gather_rows, verification only)
    and rank 0 checks every rank's rows; the result covers the whole job."""
    import oracle

    out = step_outputs(ds3, S)
    threads = cpu_cores()
    if world == 1:
        res = check_outputs(oracle.port(), table, params, make_host_set(set_seed(0, 0)), out, threads)
        res["ranks_checked"] = 1
        res["ok"] = parity_ok(res)
        return res
    import torch

    from qw3_b200.shard import gather_rows

    full = {}
    for name, a in out.items():
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        full[name] = gather_rows(t, a.shape[0] * world).cpu().numpy()
    res = {}
    if rank == 0:
        O = oracle.port()
        per = []
        for r in range(world):
            part = {n: a.reshape(world, -1, *a.shape[1:])[r] for n, a in full.items()}
            per.append(check_outputs(O, table, params, make_host_set(set_seed(0, r)), part, threads))
        for k in per[0]:
            vals = [p[k] for p in per]
            res[k] = max(vals) if k.endswith("tol_ratio") else all(vals)
        res["ranks_checked"] = world
        res["gather"] = "NCCL all_gather of every rank's step outputs (verification only, after timing setup)"
        res["ok"] = parity_ok(res)
    return res


def op_loops(ds3, P, max_over_ranks, barrier, peak, budget=320e6):
    """Average duration of each op of the step launched alone, back to back,
    rotating over n copies of its activations (n * bytes >= budget > L2).
    Copies are slices of framework-allocated device slabs (random fill on the
    device), wrapped as ds3_cuda buffers."""
    import math

    import torch

    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    out = {}
    keep = []

    def slab(shape, kind="normal", std=1.0, hi=V):
        if kind == "normal":
            t = torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std
        elif kind == "ids":
            t = torch.randint(0, hi, shape, generator=gen, device=dev, dtype=torch.int32)
        elif kind == "uniform":
            t = torch.rand(shape, generator=gen, device=dev, dtype=torch.float32)
        else:
            t = torch.empty(shape, device=dev, dtype=torch.float32)
        keep.append(t)
        return t

    def views(t, n):
        w = ds3.buffer_wrap(t.data_ptr(), t.numel() * t.element_size())
        keep.append(w)
        per = t.numel() * t.element_size() // n
        vs = [ds3.buffer_view(w, i * per, per) for i in range(n)]
        keep.extend(vs)
        return vs

    eps = I.NORM_EPS
    for op in OPS:
        n = int(min(2048, max(2, math.ceil(budget / ALGO_BYTES[op]))))
        if op == "embed_rms_norm":
            ids, hid, nrm = views(slab((n, T), "ids"), n), views(slab((n, T, H), "empty"), n), views(
                slab((n, T, H), "empty"), n)
            fns = [lambda i=i: ds3.embed_rms_norm(P["table"], ids[i], P["attn_norm"], hid[i], nrm[i], T, H, V,
                                                  ds3.TYPE_Q4_K, Q4K_ROW, eps) for i in range(n)]
        elif op == "qk_norm_rope":
            q, k = views(slab((n, T, NQ, HD)), n), views(slab((n, T, NK, HD)), n)
            pos = views(slab((n, T), "ids", hi=T), n)
            fns = [lambda i=i: ds3.qk_norm_rope(q[i], k[i], P["q_norm"], P["k_norm"], pos[i], T, NQ, NK, HD,
                                                I.ROPE_THETA, eps) for i in range(n)]
        elif op == "add_rms_norm":
            x, r = views(slab((n, T, H)), n), views(slab((n, T, H)), n)
            so, no = views(slab((n, T, H), "empty"), n), views(slab((n, T, H), "empty"), n)
            fns = [lambda i=i: ds3.add_rms_norm(x[i], r[i], P["ffn_norm"], so[i], no[i], H, T, eps) for i in range(n)]
        elif op == "router_softmax_topk":
            lg = views(slab((n, T, E), std=2.0), n)
            ix, sc = views(slab((n, T, K), "empty"), n), views(slab((n, T, K), "empty"), n)
            fns = [lambda i=i: ds3.router_softmax_topk(lg[i], None, ix[i], sc[i], T, E, K, True) for i in range(n)]
        elif op == "swiglu":
            g, u = views(slab((n, T * K, FF), std=1.5), n), views(slab((n, T * K, FF), std=1.5), n)
            w, o = views(slab((n, T * K), "uniform"), n), views(slab((n, T * K, FF), "empty"), n)
            fns = [lambda i=i: ds3.swiglu(g[i], u[i], w[i], o[i], T * K, FF) for i in range(n)]
        else:
            y, r = views(slab((n, T * K, H)), n), views(slab((n, T, H)), n)
            w, o = views(slab((n, T, K), "uniform"), n), views(slab((n, T, H), "empty"), n)
            fns = [lambda i=i: ds3.moe_combine_residual(y[i], None, w[i], r[i], o[i], T, K, H) for i in range(n)]
        torch.cuda.synchronize()
        reps = max(n, 64)
        ms = time_launches(ds3, fns, reps, max_over_ranks, barrier)
        gbs = ALGO_BYTES[op] / (ms * 1e-3) / 1e9
        out[op] = {"avg_us": round(ms * 1e3, 3), "algo_bytes": ALGO_BYTES[op], "gbs": round(gbs, 1),
                   "frac_of_measured_peak": round(gbs / peak, 4), "copies": n}
        for x in keep:
            if hasattr(x, "free"):
                x.free()
        keep.clear()
        torch.cuda.empty_cache()
    return out


def run_e2e(ds3, P, sets, hosts, steps, world, max_over_ranks, barrier):
    """Same step from pinned host memory: every input is copied host->device
    and the step's outputs read back, inside the timed region, through the
    C-ABI. Two forms:
      pipelined (the reported value): steps alternate between two device input
        sets; step i+1's inputs arrive on copy lane 1 and step i-1's results
        leave on copy lane 2 while step i computes on lane 0, ordered by
        events (ds3_cuda_lane_*);
      serial: one batch per step - copies in, the six ops, copies out."""
    import torch

    def pinned(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        return t.numpy()

    src = [{n: pinned(h[n]) for n in DevSet.IN} for h in hosts[:2]]

    def out_bufs():
        o = {"out": np.empty((T, H), np.float32), "idx": np.empty((T, K), np.int32),
             "scores": np.empty((T, K), np.float32)}
        return {n: pinned(a) for n, a in o.items()}

    outs = [out_bufs(), out_bufs()]
    h2d = sum(a.nbytes for a in src[0].values())
    d2h = sum(a.nbytes for a in outs[0].values())
    n = max(4, min(steps, 200))

    def ok(rc):
        if rc != 0:
            raise RuntimeError(ds3.last_error())

    def serial_step():
        ds3.begin_batch()
        for name, a in src[0].items():
            ok(ds3.buffer_write_async(sets[0].b[name], 0, a))
        enqueue_step(ds3, P, sets[0])
        for name, a in outs[0].items():
            ok(ds3.buffer_read_async(sets[0].b[name], 0, a))
        ok(ds3.end_batch())

    # Event slots: inputs of set s uploaded / set s computed / set s read out.
    UP, DONE, OUT = 100, 110, 120

    def pipelined(k):
        ok(ds3.begin_batch())
        for i in range(k):
            s = i % 2
            S = sets[s]
            if i >= 2:
                ok(ds3.lane_wait(1, DONE + s))  # set s's inputs are free once step i-2 has run
            for name, a in src[s].items():
                ok(ds3.lane_write(1, S.b[name], 0, a))
            ok(ds3.lane_record(1, UP + s))
            ok(ds3.lane_wait(0, UP + s))
            if i >= 2:
                ok(ds3.lane_wait(0, OUT + s))  # step i-2's results have left set s
            enqueue_step(ds3, P, S)
            ok(ds3.lane_record(0, DONE + s))
            ok(ds3.lane_wait(2, DONE + s))
            for name, a in outs[s].items():
                ok(ds3.lane_read(2, S.b[name], 0, a))
            ok(ds3.lane_record(2, OUT + s))
        ok(ds3.end_batch())

    for _ in range(3):
        serial_step()
    pipelined(4)
    # The host link is shared with whatever else the host does: its rate is
    # measured right before and right after the e2e loops, and the better of
    # the two is the roofline's denominator.
    link0 = link_peak(ds3, sets[0], src[0], outs[0], max_over_ranks, barrier)
    barrier()
    t0 = time.perf_counter()
    pipelined(n)
    el = max_over_ranks(time.perf_counter() - t0)
    barrier()
    t0 = time.perf_counter()
    for _ in range(n):
        serial_step()
    el_serial = max_over_ranks(time.perf_counter() - t0)
    barrier()
    link1 = link_peak(ds3, sets[0], src[0], outs[0], max_over_ranks, barrier)
    link = {k: max(link0[k], link1[k]) for k in link0}
    link["before_after"] = [link0, link1]
    ms = 1e3 * el / n
    # H2D and D2H use separate copy engines, so with the lanes the floor is
    # the larger of the two directions (the ops hide under the copies).
    floor_ms = 1e3 * max(h2d / (link["h2d_gbs"] * 1e9), d2h / (link["d2h_gbs"] * 1e9))
    return {"value": round(world * T * n / el, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": n, "ms_per_step": round(ms, 4),
            "copy_gbs": round((h2d + d2h) / (el / n) / 1e9, 2),
            "roofline": {"bound": "host link", "link": link, "floor_ms_per_step": round(floor_ms, 4),
                         "frac": round(floor_ms / ms, 4),
                         "note": "floor = the step's H2D bytes at the pinned H2D rate of the same copies alone (the "
                                 "D2H bytes overlap on the other copy engine), every rank copying at once; the "
                                 "better of the rates measured just before and just after the e2e loops"},
            "serial": {"value": round(world * T * n / el_serial, 1), "ms_per_step": round(1e3 * el_serial / n, 4),
                       "api": "begin_batch / 9 x buffer_write_async / 6 ops / 3 x buffer_read_async / end_batch"},
            "api": "one batch: per step, 9 x lane_write on copy lane 1, the 6 ops on lane 0, 3 x lane_read on lane 2, "
                   "two device input sets alternating, ordered by lane_record / lane_wait (wall clock)"}


def link_peak(ds3, S, src, outs, max_over_ranks, barrier):
    """Pinned host<->device copy rate of exactly the e2e step's transfers
    (its 9 input copies, then its 3 output copies, repeated on the module
    stream, wall clock, all ranks at once, slowest rank), for the e2e
    roofline."""
    h2d = sum(a.nbytes for a in src.values())
    d2h = sum(a.nbytes for a in outs.values())
    out = {}
    for name, fn, nbytes in (("h2d", lambda: [ds3.buffer_write_async(S.b[k], 0, a) for k, a in src.items()], h2d),
                             ("d2h", lambda: [ds3.buffer_read_async(S.b[k], 0, a) for k, a in outs.items()], d2h)):
        reps = max(5, int(8e9 // max(nbytes, 1)))
        for _ in range(2):
            fn()
        ds3.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(reps):
            if any(fn()):
                raise RuntimeError(ds3.last_error())
        ds3.synchronize()
        el = max_over_ranks(time.perf_counter() - t0)
        out[f"{name}_gbs"] = round(nbytes * reps / el / 1e9, 2)
    barrier()
    return out


# ------------------------------------------------------ per-config kernels
def time_launches(ds3, fns, reps, max_over_ranks, barrier):
    """Average device time of fns[i % len(fns)]() over `reps` launches, with
    warm-up, captured in one graph and timed with events on the module stream."""
    for i in range(3):
        fns[i % len(fns)]()
    ds3.synchronize()
    ds3.graph_begin()
    for i in range(reps):
        fns[i % len(fns)]()
    g = ds3.graph_end()
    ds3.graph_launch(g)
    ds3.synchronize()
    barrier()
    ds3.timer_mark(2)
    ds3.graph_launch(g)
    ds3.timer_mark(3)
    ds3.synchronize()
    ms = max_over_ranks(ds3.timer_elapsed_ms(2, 3)) / reps
    ds3.graph_free(g)
    return ms


def stream_floor(ds3, kernels, max_over_ranks, barrier):
    """Size-matched streaming floor for each step kernel: ds3_cuda_vec_add (two
    reads, one write, all loads issued first, PDL) moving the kernel's
    algorithmic bytes, timed like the kernel itself (back-to-back launches in
    one graph, operands rotated over sets that exceed L2). At T=512 every op
    fits in one wave, so even a plain stream stays below the copy peak; this is
    the time a kernel of that size could reach."""
    for op, k in kernels.items():
        nbytes = k["algo_bytes"]
        n = (nbytes // 12) // 4 * 4
        if n < 1 << 16:
            continue  # latency-bound (the router): no meaningful stream
        nsets = max(2, -(-330_000_000 // (12 * n)))
        bufs = [[ds3.empty(n * 4) for _ in range(3)] for _ in range(nsets)]
        for a, b, _ in bufs:
            ds3.buffer_zero_f32(a, n * 4)
            ds3.buffer_zero_f32(b, n * 4)
        fns = [lambda a=a, b=b, c=c: ds3.vec_add(a, b, c, n) for a, b, c in bufs]
        us = time_launches(ds3, fns, max(40, nsets), max_over_ranks, barrier) * 1e3
        k["stream_floor_us"] = round(us, 3)
        k["of_stream_floor"] = round(us / k["avg_us"], 4)
        for trio in bufs:
            for x in trio:
                x.free()


def run_rope_f16(ds3, T, max_over_ranks, barrier):
    """QK-norm + RoPE with fp16 storage on T tokens, in place, over three
    input sets (together larger than L2 from T = 8192 up)."""
    sets = []
    for i in range(3):
        q = ds3.upload(I.normal(7000 + i, (T, NQ, HD)).astype(np.float16))
        k = ds3.upload(I.normal(7100 + i, (T, NK, HD)).astype(np.float16))
        sets.append((q, k))
    qw, kw = ds3.upload(I.gamma(HD, 7200)), ds3.upload(I.gamma(HD, 7201))
    pos = ds3.upload(np.arange(T, dtype=np.int32))
    fns = [lambda q=q, k=k: ds3.qk_norm_rope(q, k, qw, kw, pos, T, NQ, NK, HD, I.ROPE_THETA, I.NORM_EPS,
                                             ds3.TYPE_F16) for q, k in sets]
    ms = time_launches(ds3, fns, 12, max_over_ranks, barrier)
    nbytes = T * (4 * (NQ + NK) * HD + 4)
    peak, _ = measured_peak()
    for b in [x for qk in sets for x in qk] + [qw, kw, pos]:
        b.free()
    return {"workload": f"qk_norm_rope_f16_T{T}", "us": round(ms * 1e3, 3), "algo_bytes": nbytes,
            "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "frac_of_measured_peak": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)}


def run_router_proj(ds3, T, max_over_ranks, barrier):
    """Router projection [T, 2048] x [128, 2048] fused with softmax/top-8,
    bit-exact sequential fp32 sums (ds3_cuda_router_logits_topk)."""
    x, w = ds3.upload(I.normal(7300, (T, H))), ds3.upload(I.normal(7301, (E, H), 0.0, 0.05))
    ix, sc = ds3.empty(T * K * 4), ds3.empty(T * K * 4)
    fns = [lambda: ds3.router_logits_topk(x, w, None, ix, sc, T, H, E, K, True)]
    ms = time_launches(ds3, fns, 20, max_over_ranks, barrier)
    for b in (x, w, ix, sc):
        b.free()
    return {"workload": f"router_logits_topk_T{T}", "us": round(ms * 1e3, 3),
            "gflops": round(2 * T * E * H / (ms * 1e-3) / 1e9, 1)}


def run_decode_ffn(ds3, T, max_over_ranks, barrier):
    """The fused decode FFN entry alone on T tokens: residual add + ffn
    RMSNorm + router projection + top-8 (ds3_cuda_add_rms_norm_router_topk)."""
    x, r = ds3.upload(I.normal(7500, (T, H))), ds3.upload(I.normal(7501, (T, H)))
    w, W = ds3.upload(I.gamma(H, 7502)), ds3.upload(I.normal(7503, (E, H), 0.0, 0.05))
    so, no = ds3.empty(T * H * 4), ds3.empty(T * H * 4)
    ix, sc = ds3.empty(T * K * 4), ds3.empty(T * K * 4)
    fns = [lambda: ds3.add_rms_norm_router_topk(x, r, w, W, so, no, None, ix, sc, T, H, E, K, I.NORM_EPS, True)]
    ms = time_launches(ds3, fns, 20, max_over_ranks, barrier)
    for b in (x, r, w, W, so, no, ix, sc):
        b.free()
    return {"workload": f"add_rms_norm_router_topk_T{T}", "us": round(ms * 1e3, 3)}


def run_expert_lists(ds3, T, max_over_ranks, barrier):
    """Device per-expert token lists for T tokens x top-8 (ds3_cuda_moe_expert_lists)."""
    lg = ds3.upload(I.normal(7400, (T, E), 0.0, 2.0))
    ix, sc = ds3.empty(T * K * 4), ds3.empty(T * K * 4)
    ds3.router_softmax_topk(lg, None, ix, sc, T, E, K, True)
    cnt, ids, gsc, slot = ds3.empty(E * 4), ds3.empty(E * T * 4), ds3.empty(E * T * 4), ds3.empty(T * K * 4)
    fns = [lambda: ds3.moe_expert_lists(ix, sc, cnt, ids, gsc, slot, T, E, K, T)]
    ms = time_launches(ds3, fns, 20, max_over_ranks, barrier)
    for b in (lg, ix, sc, cnt, ids, gsc, slot):
        b.free()
    return {"workload": f"moe_expert_lists_T{T}", "us": round(ms * 1e3, 3)}


def n_copies(set_bytes: int, budget: int = 320_000_000, lo: int = 2) -> int:
    """Input sets to rotate so a config's launches stream from HBM: together
    at least `budget` bytes (> 126 MB L2) on every rank, at any N."""
    return max(lo, -(-budget // max(set_bytes, 1)))


def run_configs(ds3, world, rank, max_over_ranks, barrier, peak, table_q4k, shard_of=0):
    """Kernel throughput on benchmark configs 2-5 (per GPU; C4/C5 rows sharded
    across the ranks). Inputs rotate over copies larger than L2 on every rank.
    Before each config is timed, its first launch (on fresh inputs) is
    compared with the oracle at the config's own size: `parity` in each entry
    (under torchrun every rank checks its shard and the flags are combined
    over ranks)."""
    import oracle

    from qw3_b200.shard import shard_range

    O = oracle.port()
    thr = cpu_cores()
    out = {}
    eps = I.NORM_EPS
    bufs = []

    def up(a):
        b = ds3.upload(a)
        bufs.append(b)
        return b

    def empty(n):
        b = ds3.empty(n)
        bufs.append(b)
        return b

    def free(*bs):
        for b in bs:
            b.free()
            if b in bufs:
                bufs.remove(b)

    def job(par: dict) -> dict:
        """Combine one rank's parity flags over all ranks (exact flags: all
        true; tolerance ratios: the worst)."""
        res = {}
        for k, v in par.items():
            if k.endswith("tol_ratio"):
                res[k] = round(max_over_ranks(float(v)), 4)
            else:
                res[k] = max_over_ranks(0.0 if v else 1.0) == 0.0
        res["ok"] = parity_ok(res)
        res["rows_checked"] = "all rows of every rank's shard"
        return res

    def rec(name, tokens, nbytes, ms, par=None, note="", copies=None):
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"tokens_per_s": round(tokens * world / (ms * 1e-3), 1), "us": round(ms * 1e3, 3),
                     "algo_bytes": nbytes, "gbs_per_gpu": round(gbs, 1),
                     "pct_of_8tbs": round(100 * gbs / NOMINAL_HBM_GBS, 2),
                     "frac_of_measured_peak": round(gbs / peak, 4)}
        if copies is not None:
            out[name]["input_copies"] = copies
        if par is not None:
            out[name]["parity"] = job(par)
        if note:
            out[name]["note"] = note

    # shard_of > 0: one GPU runs the row shard rank 0 would hold among
    # shard_of GPUs (a single-GPU look at the per-GPU sizes of a larger run).
    a, b = shard_range(32768, shard_of, 0) if shard_of else shard_range(32768, world, rank)
    n = b - a
    w = up(I.gamma(H, 3))

    # C4: add + RMSNorm on [32768, 2048], rows sharded.
    nc = n_copies(4 * n * H * 4)
    xh = [I.normal(4000 + i + 50 * rank, (n, H)) for i in range(2)]
    rh = [I.normal(4100 + i + 50 * rank, (n, H)) for i in range(2)]
    xs = [up(xh[i % 2]) for i in range(nc)]
    rs = [up(rh[i % 2]) for i in range(nc)]
    ss = [empty(n * H * 4) for _ in range(nc)]
    os_ = [empty(n * H * 4) for _ in range(nc)]
    assert ds3.add_rms_norm(xs[0], rs[0], w, ss[0], os_[0], H, n, eps) == 0, ds3.last_error()
    ws, wn = O.add_rms_norm(xh[0], rh[0], I.gamma(H, 3), eps, thr)
    par = {"sum_bitexact": bitexact(ds3.download(ss[0], np.float32, (n, H)), ws),
           "norm_tol_ratio": tol_ratio(ds3.download(os_[0], np.float32, (n, H)), wn)}
    del ws, wn
    fns = [lambda i=i: ds3.add_rms_norm(xs[i], rs[i], w, ss[i], os_[i], H, n, eps) for i in range(nc)]
    rec("c4_add_rms_norm_T32768", n, n * 4 * H * 4, time_launches(ds3, fns, max(20, nc), max_over_ranks, barrier),
        par, copies=nc)
    free(*xs, *rs)
    del xh, rh

    free(*ss, *os_)

    # C4: Q6_K embed of 32768 ids over the full vocabulary; output copies
    # rotate so the written rows exceed L2 on every rank.
    nce = n_copies(n * 2 * H * 4)
    eh = [empty(n * H * 4) for _ in range(nce)]
    eo = [empty(n * H * 4) for _ in range(nce)]
    tab6 = I.q6k_table(V, H, 4200)
    t6 = ds3.buffer_from_mmap(tab6)
    bufs.append(t6)
    idh = [I.token_ids(n, 4300 + i + 50 * rank) for i in range(nce)]
    ids = [up(x) for x in idh]
    assert ds3.embed_rows(t6, ids[0], eo[0], n, H, V, ds3.TYPE_Q6_K, 1680) == 0, ds3.last_error()
    _, want = O.embed_rows(tab6, 14, 1680, V, idh[0], H, thr)
    par = {"embed_bitexact": bitexact(ds3.download(eo[0], np.float32, (n, H)), want)}
    del want, tab6
    fns = [lambda i=i: ds3.embed_rows(t6, ids[i], eo[i], n, H, V, ds3.TYPE_Q6_K, 1680) for i in range(nce)]
    rec("c4_embed_q6k_T32768", n, n * (1680 + 4 + 4 * H),
        time_launches(ds3, fns, max(20, nce), max_over_ranks, barrier), par, copies=nce)
    free(t6)
    # Same gather with the Q4_K table and the fused attn_norm.
    t4 = ds3.buffer_from_mmap(table_q4k)
    bufs.append(t4)
    assert ds3.embed_rms_norm(t4, ids[0], w, eh[0], eo[0], n, H, V, ds3.TYPE_Q4_K, 1152, eps) == 0, ds3.last_error()
    _, wh, wn = O.embed_rms_norm(table_q4k, 12, 1152, V, idh[0], H, I.gamma(H, 3), eps, thr)
    par = {"hidden_bitexact": bitexact(ds3.download(eh[0], np.float32, (n, H)), wh),
           "norm_tol_ratio": tol_ratio(ds3.download(eo[0], np.float32, (n, H)), wn)}
    del wh, wn
    fns = [lambda i=i: ds3.embed_rms_norm(t4, ids[i], w, eh[i], eo[i], n, H, V, ds3.TYPE_Q4_K, 1152, eps)
           for i in range(nce)]
    rec("embed_q4k_rms_norm_T32768", n, n * (1152 + 4 + 8 * H),
        time_launches(ds3, fns, max(20, nce), max_over_ranks, barrier), par, copies=nce)
    free(t4, *eh, *eo, *ids)

    # C5: QK-norm + RoPE on [32768, 32/4, 128], pos 0..32767, fp32 and fp16
    # storage, in place, rotating over copies.
    pos = up(np.arange(a, b, dtype=np.int32))
    qw_h, kw_h = I.gamma(HD, 5002), I.gamma(HD, 5003)
    qw, kw = up(qw_h), up(kw_h)
    pos_h = np.arange(a, b, dtype=np.int32)
    for storage, dt, name, rtol, atol in ((0, np.float32, "c5_qk_norm_rope_f32_T32768", 1e-5, 1e-6),
                                         (1, np.float16, "c5_qk_norm_rope_f16_T32768", 2e-3, 1e-3)):
        es = np.dtype(dt).itemsize
        nc5 = n_copies(n * (NQ + NK) * HD * es, lo=1)
        qh = I.normal(5000 + 10 * storage + 50 * rank, (n, NQ, HD)).astype(dt)
        kh = I.normal(5001 + 10 * storage + 50 * rank, (n, NK, HD)).astype(dt)
        qs = [up(qh) for _ in range(nc5)]
        ks = [up(kh) for _ in range(nc5)]
        assert ds3.qk_norm_rope(qs[0], ks[0], qw, kw, pos, n, NQ, NK, HD, I.ROPE_THETA, eps, storage) == 0
        qo, ko = O.qk_norm_rope(qh.astype(np.float32), kh.astype(np.float32), qw_h, kw_h, pos_h, I.ROPE_THETA,
                                eps, thr)
        gq = ds3.download(qs[0], dt, qh.shape).astype(np.float32)
        gk = ds3.download(ks[0], dt, kh.shape).astype(np.float32)
        par = {"q_tol_ratio": tol_ratio(gq, qo, rtol, atol), "k_tol_ratio": tol_ratio(gk, ko, rtol, atol)}
        del qo, ko, gq, gk, qh, kh
        fns = [lambda i=i: ds3.qk_norm_rope(qs[i], ks[i], qw, kw, pos, n, NQ, NK, HD, I.ROPE_THETA, eps, storage)
               for i in range(nc5)]
        rec(name, n, n * (2 * es * (NQ + NK) * HD + 4), time_launches(ds3, fns, max(20, nc5), max_over_ranks, barrier),
            par, note=f"tolerance {rtol:g} rel / {atol:g} abs" + (" vs the oracle on the fp16-rounded inputs"
                                                                    if storage else ""), copies=nc5)
        free(*qs, *ks)

    # Next-row kernel: QK-norm + RoPE with the fp16 KV-cache write fused in,
    # against the two launches it replaces (qk_norm_rope + kv_cache_write_batch
    # on the rotated k and v), at the chunk size and at T=32768 (sharded).
    for tk in (512, n):
        msq = max(tk, 4096)
        # Copies of q / k / v (and their own cache pair) that together exceed
        # L2 on every rank, rotated between launches.
        nkv = n_copies(tk * (NQ + 2 * NK) * HD * 4 + 2 * msq * NK * HD * 2)
        qh5, kh5, vh5 = I.normal(5100, (tk, NQ, HD)), I.normal(5101, (tk, NK, HD)), I.normal(5102, (tk, NK, HD))
        sets5 = []
        for _ in range(nkv):
            sets5.append((up(qh5), up(kh5), up(vh5), empty(msq * NK * HD * 2), empty(msq * NK * HD * 2)))
        pk = up(np.arange(tk, dtype=np.int32))
        fused = [lambda s5=s5: ds3.qk_norm_rope_kv(s5[0], s5[1], s5[2], qw, kw, pk, s5[3], s5[4], tk, NQ, NK, HD, msq,
                                                   I.ROPE_THETA, eps) for s5 in sets5]
        fb = tk * (8 * (NQ + NK) * HD + 4 + 4 * NK * HD + 2 * 2 * NK * HD)
        rec(f"qk_norm_rope_kv_write_T{tk}", tk, fb, time_launches(ds3, fused, max(20, nkv), max_over_ranks, barrier),
            note="fused: q/k in place + fp16 K/V cache rows", copies=nkv)

        def two(s5):
            ds3.qk_norm_rope(s5[0], s5[1], qw, kw, pk, tk, NQ, NK, HD, I.ROPE_THETA, eps)
            ds3.kv_cache_write_batch(s5[1], s5[2], s5[3], s5[4], 0, tk, msq, NQ, NK, HD)

        rec(f"qk_norm_rope_then_kv_write_T{tk}", tk, fb,
            time_launches(ds3, [lambda s5=s5: two(s5) for s5 in sets5], max(20, nkv), max_over_ranks, barrier),
            note="unfused reference sequence, same algorithmic bytes", copies=nkv)
        free(pk, *[b for s5 in sets5 for b in s5])

    # Next-row kernel: device-side per-expert token lists for a 512-token
    # chunk (replaces the host loop + per-layer index readback of the engine).
    lg_r = I.normal(5200, (512, E), 0.0, 2.0)
    ixr, scr = up(np.zeros((512, K), np.int32)), up(np.zeros((512, K), np.float32))
    ds3.router_softmax_topk(up(lg_r), None, ixr, scr, 512, E, K, True)
    cnt, lids, lsc, slot = empty(E * 4), empty(E * 512 * 4), empty(E * 512 * 4), empty(512 * K * 4)
    fn = [lambda: ds3.moe_expert_lists(ixr, scr, cnt, lids, lsc, slot, 512, E, K, 512)]
    rec("moe_expert_lists_T512", 512, 512 * K * (4 + 4 + 4 + 4 + 4), time_launches(ds3, fn, 20, max_over_ranks, barrier),
        note="latency-bound permutation, one CTA per expert; bytes: idx, scores in; ids, scores, slot out")

    # Next-row kernel: router projection (sequential fp32 dot products in the
    # reference's order, CUDA cores) fused with softmax/top-8, 512 tokens.
    xr_ = up(I.normal(5300, (512, H)))
    wr_ = up(I.normal(5301, (E, H), 0.0, 0.05))
    fn = [lambda: ds3.router_logits_topk(xr_, wr_, None, ixr, scr, 512, H, E, K, True)]
    us_r = time_launches(ds3, fn, 20, max_over_ranks, barrier)
    rec("router_logits_topk_T512", 512, 512 * (4 * H + 64) + E * H * 4, us_r,
        note="bit-exact sequential fp32 projection: %.0f GFLOP/s on CUDA cores" % (2 * 512 * E * H / (us_r * 1e-3) / 1e9))

    run_c1_c3(ds3, O, thr, rec, up, empty, free, table_q4k, max_over_ranks, barrier)
    run_c2(ds3, O, thr, rec, up, empty, w, qw, kw, qw_h, kw_h, max_over_ranks, barrier)

    for x in list(bufs):
        x.free()
    return out


def run_c1_c3(ds3, O, thr, rec, up, empty, free, table_q4k, max_over_ranks, barrier):
    """Benchmark configs 1 and 3 on their own (the timed step contains both):
      C1: layer-0 pre-attention chain on a 512-token chunk - Q4_K gather +
          attn_norm, then QK-norm + RoPE at positions 0..511 (2 launches);
      C3: routed-expert block - router softmax/top-8 on [512, 128], SwiGLU x
          routing weight on [4096, 768], weighted combine + residual into
          [512, 2048] (3 launches).
    Inputs rotate over copies larger than L2; the first chain of each is
    compared with the oracle."""
    eps = I.NORM_EPS
    par_h = make_params()
    params = {k: up(v) for k, v in par_h.items()}
    t4 = ds3.buffer_from_mmap(table_q4k)
    # C1
    c1_in = T * (4 + 4 * NQ * HD + 4 * NK * HD)
    nc = n_copies(c1_in + 2 * T * H * 4)
    hosts = [make_host_set(7000 + 13 * i) for i in range(2)]
    sets = []
    for i in range(nc):
        hi = hosts[i % 2]
        sets.append({"ids": up(hi["ids"]), "q": up(hi["q"]), "k": up(hi["k"]), "pos": up(hi["pos"]),
                     "hid": empty(T * H * 4), "nrm": empty(T * H * 4)})

    def c1(S):
        ds3.embed_rms_norm(t4, S["ids"], params["attn_norm"], S["hid"], S["nrm"], T, H, V, ds3.TYPE_Q4_K, Q4K_ROW, eps)
        ds3.qk_norm_rope(S["q"], S["k"], params["q_norm"], params["k_norm"], S["pos"], T, NQ, NK, HD, I.ROPE_THETA,
                         eps)

    c1(sets[0])
    ds3.synchronize()
    h = hosts[0]
    _, wh, wn = O.embed_rms_norm(table_q4k, 12, Q4K_ROW, V, h["ids"], H, par_h["attn_norm"], eps, thr)
    qo, ko = O.qk_norm_rope(h["q"], h["k"], par_h["q_norm"], par_h["k_norm"], h["pos"], I.ROPE_THETA, eps, thr)
    par = {"hidden_bitexact": bitexact(ds3.download(sets[0]["hid"], np.float32, (T, H)), wh),
           "norm_tol_ratio": tol_ratio(ds3.download(sets[0]["nrm"], np.float32, (T, H)), wn),
           "qk_rope_tol_ratio": max(tol_ratio(ds3.download(sets[0]["q"], np.float32, qo.shape), qo),
                                    tol_ratio(ds3.download(sets[0]["k"], np.float32, ko.shape), ko))}
    c1_bytes = ALGO_BYTES["embed_rms_norm"] + ALGO_BYTES["qk_norm_rope"]
    rec("c1_layer0_pre_T512", T, c1_bytes,
        time_launches(ds3, [lambda S=S: c1(S) for S in sets], max(20, nc), max_over_ranks, barrier), par,
        note="Q4_K gather + attn_norm, then QK-norm + RoPE: 2 dependent launches", copies=nc)
    free(t4, *[b for S in sets for b in S.values()])

    # C3
    c3_bytes = ALGO_BYTES["router_softmax_topk"] + ALGO_BYTES["swiglu"] + ALGO_BYTES["moe_combine_residual"]
    nc = n_copies(c3_bytes)
    sets = []
    for i in range(nc):
        hi = hosts[i % 2]
        sets.append({"logits": up(hi["logits"]), "gate": up(hi["gate"]), "up": up(hi["up"]), "y": up(hi["y"]),
                     "res": up(hi["attn_out"]), "idx": empty(T * K * 4), "sc": empty(T * K * 4),
                     "act": empty(T * K * FF * 4), "out": empty(T * H * 4)})

    def c3(S):
        ds3.router_softmax_topk(S["logits"], None, S["idx"], S["sc"], T, E, K, True)
        ds3.swiglu(S["gate"], S["up"], S["sc"], S["act"], T * K, FF)
        ds3.moe_combine_residual(S["y"], None, S["sc"], S["res"], S["out"], T, K, H)

    c3(sets[0])
    ds3.synchronize()
    h = hosts[0]
    _, iw, sw = O.router(h["logits"], K, True, thr)
    got_sc = ds3.download(sets[0]["sc"], np.float32, (T, K))
    par = {"top8_exact": bitexact(ds3.download(sets[0]["idx"], np.int32, (T, K)), iw),
           "scores_tol_ratio": tol_ratio(got_sc, sw),
           "swiglu_tol_ratio": tol_ratio(ds3.download(sets[0]["act"], np.float32, (T * K, FF)),
                                         O.swiglu(h["gate"], h["up"], got_sc.reshape(-1), thr)),
           "combine_bitexact": bitexact(ds3.download(sets[0]["out"], np.float32, (T, H)),
                                        O.combine(h["y"], got_sc, h["attn_out"], None, thr))}
    rec("c3_routed_expert_T512", T, c3_bytes,
        time_launches(ds3, [lambda S=S: c3(S) for S in sets], max(20, nc), max_over_ranks, barrier), par,
        note="router softmax/top-8, SwiGLU x routing weight, combine + residual: 3 dependent launches "
             "(y [4096, 2048] stands in for the out-of-scope down projection)", copies=nc)
    free(*[b for S in sets for b in S.values()], *params.values())


def run_c2(ds3, O, thr, rec, up, empty, w, qw, kw, qw_h, kw_h, max_over_ranks, barrier):
    """C2: a decode batch of 64 tokens through 48 layers (independent seeded
    inputs per layer): add + ffn RMSNorm [64, 2048], QK-norm + RoPE
    [64, 32/4, 128], router softmax/top-8 [64, 128] per layer, then the final
    RMSNorm. Two launch structures over the same inputs:
      layer grid: the per-layer inputs are independent, so each op runs once
                  over all 48 x 64 rows (4 launches per pass) - the config's
                  number;
      chain:      the engine's dependent order, 3 launches per layer plus the
                  final norm (145 launches), what a layer-by-layer engine sees.
    Parity: the first layer-grid pass against the oracle on every layer."""
    eps = I.NORM_EPS
    L, B2 = 48, 64
    R = L * B2
    hid_h, res_h = I.normal(6000, (R, H)), I.normal(6001, (R, H))
    q_h, k_h = I.normal(6002, (R, NQ, HD)), I.normal(6003, (R, NK, HD))
    lg_h = I.normal(6004, (R, E), 0, 2)
    pos_h = np.tile(I.rng(6005).integers(0, 4096, B2).astype(np.int32), L)
    hid, res, q2, k2, lg = up(hid_h), up(res_h), up(q_h), up(k_h), up(lg_h)
    nrm, ix, sc = empty(R * H * 4), empty(R * K * 4), empty(R * K * 4)
    fin = empty(B2 * H * 4)
    pos2 = up(pos_h)
    last = ds3.buffer_view(hid, (L - 1) * B2 * H * 4, B2 * H * 4)
    sum_out = empty(R * H * 4)

    def grid_pass():
        ds3.add_rms_norm(hid, res, w, sum_out, nrm, H, R, eps)
        ds3.qk_norm_rope(q2, k2, qw, kw, pos2, R, NQ, NK, HD, I.ROPE_THETA, eps)
        ds3.router_softmax_topk(lg, None, ix, sc, R, E, K, True)
        ds3.rms_norm(last, w, fin, H, B2, eps)

    grid_pass()
    ds3.synchronize()
    w_h = I.gamma(H, 3)
    s_want, n_want = O.add_rms_norm(hid_h, res_h, w_h, eps, thr)
    qo, ko = O.qk_norm_rope(q_h, k_h, qw_h, kw_h, pos_h, I.ROPE_THETA, eps, thr)
    _, iw, sw = O.router(lg_h, K, True, thr)
    fw = O.rms_norm_rows(hid_h[(L - 1) * B2:], w_h, eps, thr)
    par = {"sum_bitexact": bitexact(ds3.download(sum_out, np.float32, (R, H)), s_want),
           "ffn_norm_tol_ratio": tol_ratio(ds3.download(nrm, np.float32, (R, H)), n_want),
           "qk_rope_tol_ratio": max(tol_ratio(ds3.download(q2, np.float32, q_h.shape), qo),
                                    tol_ratio(ds3.download(k2, np.float32, k_h.shape), ko)),
           "top8_exact": bitexact(ds3.download(ix, np.int32, (R, K)), iw),
           "scores_tol_ratio": tol_ratio(ds3.download(sc, np.float32, (R, K)), sw),
           "final_norm_tol_ratio": tol_ratio(ds3.download(fin, np.float32, (B2, H)), fw)}
    c2_bytes = B2 * L * (32768 + 36868 + 576) + B2 * 16384
    ms = time_launches(ds3, [grid_pass], 10, max_over_ranks, barrier)
    rec("c2_decode_B64_x48_layers", B2, c2_bytes, ms, par,
        note="layer grid: 4 launches per 48-layer pass (each op over all 48 x 64 rows; the per-layer inputs are "
             "independent); tokens_per_s counts one 48-layer pass per token")

    views = []

    def view(buf, i, per):
        v = ds3.buffer_view(buf, i * per, per)
        views.append(v)
        return v

    def chain():
        for l in range(L):
            ds3.add_rms_norm(view(hid, l, B2 * H * 4), view(res, l, B2 * H * 4), w, view(sum_out, l, B2 * H * 4),
                             view(nrm, l, B2 * H * 4), H, B2, eps)
            ds3.qk_norm_rope(view(q2, l, B2 * NQ * HD * 4), view(k2, l, B2 * NK * HD * 4), qw, kw,
                             view(pos2, l, B2 * 4), B2, NQ, NK, HD, I.ROPE_THETA, eps)
            ds3.router_softmax_topk(view(lg, l, B2 * E * 4), None, view(ix, l, B2 * K * 4), view(sc, l, B2 * K * 4),
                                    B2, E, K, True)
        ds3.rms_norm(last, w, fin, H, B2, eps)

    ms = time_launches(ds3, [chain], 3, max_over_ranks, barrier)
    rec("c2_decode_B64_x48_layers_chain", B2, c2_bytes, ms,
        note="the engine's layer-by-layer order: 3 dependent launches per layer + final norm = 145 launches")

    # The engine-faithful decode layer in 2 launches: QK-norm + RoPE, then
    # residual add + ffn_norm + router projection (a seeded fp32 router
    # weight per layer, N(0, 0.05)) + top-8 in one kernel; the router input
    # is the normed hidden state, as in forward_layer_pre
    # (src/ds3_engine.c:508-535), so the config's given logits are not used.
    wr_h = [I.normal(6100 + l, (E, H), 0.0, 0.05) for l in range(L)]
    wr = [up(a) for a in wr_h]

    def chain2():
        for l in range(L):
            ds3.qk_norm_rope(view(q2, l, B2 * NQ * HD * 4), view(k2, l, B2 * NK * HD * 4), qw, kw,
                             view(pos2, l, B2 * 4), B2, NQ, NK, HD, I.ROPE_THETA, eps)
            ds3.add_rms_norm_router_topk(view(hid, l, B2 * H * 4), view(res, l, B2 * H * 4), w, wr[l],
                                         view(sum_out, l, B2 * H * 4), view(nrm, l, B2 * H * 4), None,
                                         view(ix, l, B2 * K * 4), view(sc, l, B2 * K * 4), B2, H, E, K, eps, True)
        ds3.rms_norm(last, w, fin, H, B2, eps)

    chain2()
    ds3.synchronize()
    # Parity of the fused entry on layers 0 and 47: sum exact, normed rows
    # within tolerance, top-8 exact against the oracle's projection of the
    # kernel's normed rows.
    par = {}
    got_s = ds3.download(sum_out, np.float32, (R, H))
    got_n_all = ds3.download(nrm, np.float32, (R, H))
    got_i = ds3.download(ix, np.int32, (R, K))
    for l in (0, L - 1):
        rows = slice(l * B2, (l + 1) * B2)
        s_w, n_w = O.add_rms_norm(hid_h[rows], res_h[rows], w_h, eps, thr)
        got_n = np.ascontiguousarray(got_n_all[rows])
        _, iw2, _ = O.router(O.router_logits(got_n, wr_h[l], thr), K, True, thr)
        par[f"l{l}_sum_bitexact"] = bitexact(np.ascontiguousarray(got_s[rows]), s_w)
        par[f"l{l}_norm_tol_ratio"] = tol_ratio(got_n, n_w)
        par[f"l{l}_top8_exact"] = bitexact(np.ascontiguousarray(got_i[rows]), iw2)
    c2f_bytes = B2 * L * (32768 + 36868 + 64) + L * E * H * 4 + B2 * 16384
    ms = time_launches(ds3, [chain2], 3, max_over_ranks, barrier)
    rec("c2_decode_B64_x48_layers_chain_fused_router", B2, c2f_bytes, ms, par,
        note="engine-faithful decode layer in 2 launches (qk_norm_rope; add_rms_norm_router_topk with the router "
             "projection from a 1 MB fp32 weight per layer) + final norm = 97 launches; bytes include the router "
             "weights")
    for v in views + [last]:
        v.free()


if __name__ == "__main__":
    sys.exit(main())
