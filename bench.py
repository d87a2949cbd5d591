"""Benchmark of the fused layer-op chain (small-vLLM's per-layer, token-row-parallel ops).

One step is one pass of the chain over the workload's token rows:
    embedding gather -> add + RMSNorm -> Qwen3 q/k RMSNorm + RoPE -> SiLU(gate) * up
each op on its own seeded synthetic inputs of the Qwen3-0.6B shapes (hidden 1024, 16/8 heads of
128, intermediate 3072, vocab 151936). The default workload is the 1,048,576-token bandwidth
sweep, token rows split evenly over the GPUs (strong scaling, no collective on the timed path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Prints ONE JSON line on rank 0. `value` is the whole-job algorithmic HBM GB/s of the chain
(bytes every op must read and write, summed over ranks, over the slowest rank's device time);
`e2e` is the same metric through svllm_ops with pinned host buffers, copies in the timed region.
`--impl reference` times the reference's CPU path on this host's cores instead (the reference's
own OpenMP rms_norm built from its sources, and the C/OpenMP restatement for the ops it lacks).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "small-vllm_b200" / "python"), str(ROOT / "oracle")]

METRIC = "fused layer-op achieved HBM GB/s (% of B200 peak) and tokens/s at 1/2/4/8 GPUs"
NOMINAL_HBM_GBS = 8000.0  # B200 HBM3e, nominal
UNIT = "GB/s"

QWEN3 = dict(name="qwen3-0.6b", hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=3072,
             vocab=151936, eps=1e-6, theta=1e6, qk_norm=True, scaling=None)
# Llama-3.2-1B with llama3 rope scaling at factor 32 (the model's config.json has 8.0; the
# formula is the same and both are tested)
LLAMA = dict(name="llama-3.2-1b", hidden=2048, heads=32, kv_heads=8, head_dim=64, inter=8192,
             vocab=128256, eps=1e-5, theta=5e5, qk_norm=False, scaling=(32.0, 1.0, 4.0, 8192))

# Algorithmic bytes per token of each op (bf16 activations; int32 ids; int64 positions):
#   embedding     read the table row and write the output row, plus the id
#   add_rms_norm  read x and residual, write residual' and the normed x
#   qk_norm_rope  read and write q (16 x 128) and k (8 x 128) in place, plus the position
#   silu_and_mul  read gate and up, write out
def op_bytes(cfg: dict, elem: int = 2) -> dict[str, int]:
    """Bytes per token of each op, activations of `elem` bytes (2: bf16, 4: fp32)."""
    h, hd, inter = cfg["hidden"], cfg["head_dim"], cfg["inter"]
    heads = cfg["heads"] + cfg["kv_heads"]
    kv_row = cfg["kv_heads"] * hd * elem
    rotary = 2 * heads * hd * elem + 8
    if cfg.get("kv_cache"):
        rotary += kv_row + 2 * kv_row + 8  # k into the cache; v read and written; the slot
    return {
        "embedding": 2 * h * elem + 4,
        "add_rms_norm": 4 * h * elem,
        rotary_op(cfg): rotary,
        "silu_and_mul": 3 * inter * elem,
    }


OPS = ["embedding", "add_rms_norm", "qk_norm_rope", "silu_and_mul"]
WORKLOADS = {
    # name: (model, total tokens, positions): positions ("uniform", hi) draw each token's
    # position from [0, hi); ("packed", n) are sequences of n tokens at positions 0..n-1;
    # ("sequences", count, lo, hi) are `count` sequences of seeded lengths in [lo, hi], packed,
    # each at positions 0..len-1 (the total is their summed length)
    "sweep": (QWEN3, 1_048_576, ("uniform", 32768)),
    "prefill": (QWEN3, None, ("sequences", 64, 128, 2048)),
    "decode": (QWEN3, 256, ("uniform", 4096)),
    "llama": (LLAMA, 16_384, ("packed", 2048)),
}


def sequence_lengths(pos_spec: tuple):
    """The seeded sequence lengths of a ("sequences", count, lo, hi) workload."""
    import numpy as np

    _, count, lo, hi = pos_spec
    return np.random.default_rng(2025).integers(lo, hi + 1, count)


def workload_total(name: str, override: int = 0) -> int:
    cfg, total, pos_spec = WORKLOADS[name]
    if override:
        return override
    return int(sequence_lengths(pos_spec).sum()) if total is None else total


def global_positions(pos_spec: tuple, total: int):
    """Positions of every token of a "packed" or "sequences" workload (numpy int64)."""
    import numpy as np

    if pos_spec[0] == "packed":
        return np.arange(total, dtype=np.int64) % pos_spec[1]
    lengths = sequence_lengths(pos_spec)
    pos = np.concatenate([np.arange(n, dtype=np.int64) for n in lengths])
    reps = -(-total // pos.size)  # a --tokens override beyond the sequences repeats them
    return np.tile(pos, reps)[:total]


def positions_label(pos_spec: tuple) -> str:
    if pos_spec[0] == "uniform":
        return f"uniform [0, {pos_spec[1]})"
    if pos_spec[0] == "packed":
        return f"sequences of {pos_spec[1]}, positions 0..{pos_spec[1] - 1}"
    return (f"{pos_spec[1]} sequences of seeded lengths in [{pos_spec[2]}, {pos_spec[3]}], "
            "packed, each at positions 0..len-1")


def rotary_op(cfg: dict) -> str:
    """Llama has no q/k norm, so its rotary step is rope alone; with a KV cache the step also
    writes the cache."""
    name = "qk_norm_rope" if cfg["qk_norm"] else "rope"
    return name + "_cache" if cfg.get("kv_cache") else name


def op_names(cfg: dict) -> list[str]:
    return [rotary_op(cfg) if op == "qk_norm_rope" else op for op in OPS]


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload",
                   choices=sorted(WORKLOADS) + ["sampling", "lm-head", "model-decode",
                                                "decode-attention", "decode-linear", "rms-norm"],
                   default="sweep",
                   help="sampling: greedy argmax over [tokens, 151936] bf16 logits (one op, "
                        "not the chain); lm-head: the tied LM head fused with greedy sampling "
                        "(one tcgen05 kernel) beside matmul + argmax; model-decode: Qwen3-0.6B "
                        "decode steps through the model forward, eager and from CUDA graphs; "
                        "decode-attention: the paged decode-attention kernel of one Qwen3-0.6B "
                        "layer beside the gather + SDPA composite it replaces; decode-linear: "
                        "the Qwen3-0.6B projections at decode batch sizes, the decode-linear "
                        "kernel beside torch.matmul (cuBLAS); rms-norm: svllm_ops.rms_norm, or "
                        "with --impl reference the reference's own CUDA rms_norm, at "
                        "1M x 1024, 16384 x 2048 and 16M x 128")
    p.add_argument("--batches", default="1,8,64,256",
                   help="model-decode: comma-separated decode batch sizes")
    p.add_argument("--context", type=int, default=512,
                   help="model-decode, decode-attention: KV-cache tokens per request")
    p.add_argument("--tokens", type=int, default=0, help="override total tokens")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer measurement")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-validate", action="store_true")
    p.add_argument("--no-configs", action="store_true",
                   help="skip the benchmark definition's configs 0-3 (measured at N=1 beside "
                        "the sweep)")
    p.add_argument("--cpu-sample-tokens", type=int, default=131072,
                   help="token rows of the cpu_baseline sample in the GPU arm's line")
    p.add_argument("--reference-tokens", type=int, default=0,
                   help="--impl reference: token rows per timed pass (default: the workload's "
                        "full count, the GPU arm's configuration)")
    p.add_argument("--kv-cache", action="store_true",
                   help="the rotary step also writes k and v into a paged KV cache "
                        "(qk_norm_rope_cache / rope_cache)")
    p.add_argument("--graph", action="store_true",
                   help="capture the chain in a CUDA graph and time replays (small-T regime)")
    return p.parse_args()


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {"hbm_gbs": 6650.0, "fallback": True}


def split_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced row range [begin, end) of `rank`."""
    base, rem = divmod(total, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


# ---------------------------------------------------------------------------------------------
# Synthetic inputs (seeded, per rank)

def make_inputs(T: int, pos_spec: tuple, cfg: dict, device, seed: int, first_row: int = 0):
    """Per-rank activations from `seed`; the weights (embedding table, norm weights) from one
    fixed seed, so every rank holds the same replicated model weights."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    gw = torch.Generator(device=device).manual_seed(1234)

    def randn(*shape, scale=1.0, shift=0.0, gen=g):
        t = torch.empty(shape, device=device, dtype=torch.bfloat16)
        return t.normal_(shift, scale, generator=gen) if shape[0] else t

    h, hd = cfg["hidden"], cfg["head_dim"]
    return {
        "table": randn(cfg["vocab"], h, scale=0.02, gen=gw),
        "w": randn(h, scale=0.1, shift=1.0, gen=gw),
        "qw": randn(hd, scale=0.1, shift=1.0, gen=gw),
        "kw": randn(hd, scale=0.1, shift=1.0, gen=gw),
        "ids": torch.randint(0, cfg["vocab"], (T,), device=device, dtype=torch.int32, generator=g),
        "x": randn(T, h),
        "residual": randn(T, h),
        "q": randn(T, cfg["heads"], hd),
        "k": randn(T, cfg["kv_heads"], hd),
        "pos": (torch.randint(0, pos_spec[1], (T,), device=device, dtype=torch.int64, generator=g)
                if pos_spec[0] == "uniform" else
                torch.from_numpy(global_positions(pos_spec, first_row + T)[first_row:]).to(device)),
        "gate": randn(T, cfg["inter"]),
        "up": randn(T, cfg["inter"]),
        **(kv_inputs(T, cfg, device, g) if cfg.get("kv_cache") else {}),
    }


def kv_inputs(T: int, cfg: dict, device, g):
    """v rows and a paged KV cache of 16-token blocks handed out in a random order, as an
    allocator would after some churn; slot_mapping follows the blocks."""
    import torch

    block = 16
    num_blocks = (T + block - 1) // block
    perm = torch.randperm(num_blocks, device=device, generator=g)
    t = torch.arange(T, device=device)
    shape = (num_blocks * block, cfg["kv_heads"], cfg["head_dim"])
    return {
        "v": torch.empty(T, cfg["kv_heads"], cfg["head_dim"], device=device,
                         dtype=torch.bfloat16).normal_(generator=g),
        "slots": perm[t // block] * block + t % block,
        "k_cache": torch.zeros(shape, device=device, dtype=torch.bfloat16),
        "v_cache": torch.zeros(shape, device=device, dtype=torch.bfloat16),
    }


class Chain:
    """The four ops through svllm_ops (LibTorch op layer -> C ABI -> sm_100a kernels)."""

    def __init__(self, inp: dict, cfg: dict):
        import torch
        import svllm_ops

        self.ops = svllm_ops
        self.inp = inp
        self.cfg = cfg
        T = inp["ids"].shape[0]
        self.emb_out = torch.empty(T, cfg["hidden"], device=inp["ids"].device, dtype=torch.bfloat16)
        self.silu_out = torch.empty(T, cfg["inter"], device=inp["ids"].device, dtype=torch.bfloat16)

    def run_op(self, name: str) -> None:
        i, c, o = self.inp, self.cfg, self.ops
        if name == "embedding":
            self.emb_out = o.embedding(i["ids"], i["table"])
        elif name == "add_rms_norm":
            o.add_rms_norm(i["x"], i["residual"], i["w"], c["eps"])
        elif name == "qk_norm_rope":
            o.qk_norm_rope(i["q"], i["k"], i["qw"], i["kw"], i["pos"], c["eps"], c["theta"],
                           scaling_of(c))
        elif name == "rope":
            o.rope(i["q"], i["k"], i["pos"], c["theta"], scaling_of(c))
        elif name == "qk_norm_rope_cache":
            o.qk_norm_rope_cache(i["q"], i["k"], i["v"], i["qw"], i["kw"], i["pos"], i["slots"],
                                 i["k_cache"], i["v_cache"], c["eps"], c["theta"], scaling_of(c))
        elif name == "rope_cache":
            o.rope_cache(i["q"], i["k"], i["v"], i["pos"], i["slots"], i["k_cache"],
                         i["v_cache"], c["theta"], scaling_of(c))
        else:
            self.silu_out = o.silu_and_mul(i["gate"], i["up"])


def scaling_of(cfg: dict):
    import svllm_ops

    return svllm_ops.Llama3RopeScaling(*cfg["scaling"]) if cfg["scaling"] else None


# ---------------------------------------------------------------------------------------------
# Clocks sampled during the timed region

class ClockSampler:
    """Samples SM clocks and clock-event reasons of the given GPUs during the timed region, from
    a thread polling NVML every few milliseconds (the timed region can be shorter than
    nvidia-smi's sampling interval). Reads settings only; changes nothing."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpus: list[int], enabled: bool = True, period_s: float = 0.005):
        self.gpus = gpus
        self.enabled = enabled
        self.period = period_s
        self.samples: list[tuple[int, float, float, int]] = []
        self._stop = None
        self._ready = None
        self._thread = None

    def _poll(self):
        import pynvml

        handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in self.gpus]
        reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._stop.is_set():
            for i, h in zip(self.gpus, handles):
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = reasons_fn(h)
                    self.samples.append((i, float(sm), float(mx), int(rs)))
                except pynvml.NVMLError:
                    pass
            self._ready.set()
            self._stop.wait(self.period)

    def __enter__(self):
        if not self.enabled:
            return self
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
        except Exception:  # NVML missing: report no samples rather than fail the bench
            return self
        self._stop = threading.Event()
        self._ready = threading.Event()
        self._thread = threading.Thread(target=self._poll, daemon=True)
        self._thread.start()
        # the timed region can be shorter than the thread's NVML set-up: start it once polling runs
        self._ready.wait(timeout=2.0)
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        for _, _, _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in self.samples),
                "sm_max_mhz": max(s[2] for s in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "NVML, polled every 5 ms"}


# ---------------------------------------------------------------------------------------------
# The CPU path (the reference arm and the cpu_baseline): the reference's own OpenMP rms_norm
# (built from its sources into oracle/_ref) where the reference has the op, and the C/OpenMP
# restatement (oracle/) for the rest. Host-resident, all host threads.

def synthetic_bf16(rng, n: int, scale: float = 1.0, shift: float = 0.0, block: int = 1 << 24):
    """n bf16 values (uint16 bits) ~ N(shift, scale^2): one seeded block of up to 16M values,
    repeated. The repeat period (32 MB) is beyond any CPU cache, so a timed pass over the array
    does the same work as over fully independent values, and 1M-token inputs take seconds to
    make instead of minutes."""
    import numpy as np

    import oracle

    base = oracle.f32_to_bf16(rng.standard_normal(min(n, block), dtype=np.float32) * scale + shift)
    out = np.empty(n, dtype=np.uint16)
    for start in range(0, n, base.size):
        m = min(base.size, n - start)
        out[start:start + m] = base[:m]
    return out


def cpu_chain_sample(tokens: int, cfg: dict, pos_spec: tuple, steps: int,
                     min_seconds: float = 0.0):
    """Times `steps` passes of the chain on host memory over `tokens` token rows, with every
    host thread: the reference's own OpenMP rms_norm (oracle/_ref) for the norms after a LibTorch
    add that updates the residual in place, as add_rms_norm does, and the C/OpenMP restatement
    for the ops the reference lacks, writing into preallocated outputs."""
    import numpy as np
    import torch

    import oracle

    cores = len(os.sched_getaffinity(0))
    # torchrun exports OMP_NUM_THREADS=1: both OpenMP pools get the cores this line reports
    torch.set_num_threads(cores)
    threads = oracle.set_num_threads(cores)
    ref = oracle.reference_module()
    rng = np.random.default_rng(1234)
    h, hd, inter = cfg["hidden"], cfg["head_dim"], cfg["inter"]

    def bf16(*shape, scale=1.0, shift=0.0):
        return synthetic_bf16(rng, int(np.prod(shape)), scale, shift).reshape(shape)

    table = bf16(cfg["vocab"], h, scale=0.02)
    ids = rng.integers(0, cfg["vocab"], tokens, dtype=np.int32)
    x, r, w = bf16(tokens, h), bf16(tokens, h), bf16(h, scale=0.1, shift=1.0)
    q, k = bf16(tokens, cfg["heads"], hd), bf16(tokens, cfg["kv_heads"], hd)
    qw, kw = bf16(hd, scale=0.1, shift=1.0), bf16(hd, scale=0.1, shift=1.0)
    pos = (rng.integers(0, pos_spec[1], tokens, dtype=np.int64) if pos_spec[0] == "uniform"
           else global_positions(pos_spec, tokens))
    gate, up = bf16(tokens, inter), bf16(tokens, inter)
    emb_out = np.empty((tokens, h), dtype=np.uint16)
    silu_out = np.empty((tokens, inter), dtype=np.uint16)
    emb_out.fill(0)
    silu_out.fill(0)  # first-touch the outputs outside the timed passes
    inv = oracle.inv_freq(cfg["theta"], hd, cfg["scaling"])
    names = op_names(cfg)

    def as_t(a):
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)

    tx, tr, tw, tq, tk = as_t(x), as_t(r), as_t(w), as_t(q), as_t(k)
    tqw, tkw = as_t(qw), as_t(kw)
    per_op = {op: 0.0 for op in names}
    done = 0
    t_start = time.perf_counter()
    while done < steps or time.perf_counter() - t_start < min_seconds:
        t0 = time.perf_counter()
        oracle.embedding(ids, table, out=emb_out)
        t1 = time.perf_counter()
        if ref is not None:
            tr.add_(tx)  # residual <- x + residual (LibTorch), then the reference's rms_norm
            ref.rms_norm(tr, tw, cfg["eps"])
        else:
            oracle.add_rms_norm(x, r, w, cfg["eps"], inplace=True)
        t2 = time.perf_counter()
        if not cfg["qk_norm"]:
            oracle.rope(q, k, pos, inv, inplace=True)
        elif ref is not None:
            qn = ref.rms_norm(tq.view(-1, hd), tqw, cfg["eps"])
            kn = ref.rms_norm(tk.view(-1, hd), tkw, cfg["eps"])
            oracle.rope(qn.view(torch.int16).numpy().view(np.uint16).reshape(q.shape),
                        kn.view(torch.int16).numpy().view(np.uint16).reshape(k.shape), pos, inv,
                        inplace=True)
        else:
            oracle.qk_norm_rope(q, k, qw, kw, pos, cfg["eps"], inv, inplace=True)
        t3 = time.perf_counter()
        oracle.silu_and_mul(gate, up, out=silu_out)
        t4 = time.perf_counter()
        for op, dt in zip(names, (t1 - t0, t2 - t1, t3 - t2, t4 - t3)):
            per_op[op] += dt
        done += 1
    nbytes = op_bytes(cfg)
    total_s = sum(per_op.values())
    gbs = sum(nbytes.values()) * tokens * done / total_s / 1e9
    kind = "reference" if ref is not None else "port"
    sample = (f"{tokens} tokens x {done} passes of the chain on host memory, {threads} OpenMP "
              "threads; "
              + ("reference's own OpenMP rms_norm (oracle/_ref, built from its sources) for the "
                 "norms, after a LibTorch add into the residual; C/OpenMP restatement (oracle/) "
                 "for embedding, rope, silu_and_mul" if ref is not None
                 else "C/OpenMP restatement (oracle/)"))
    ops = {op: round(nbytes[op] * tokens * done / per_op[op] / 1e9, 2) for op in names}
    return {"value": round(gbs, 2), "unit": UNIT, "cores": cores, "kind": kind, "sample": sample,
            "ops_gbs": ops, "tokens_per_s": round(tokens * done / total_s, 1),
            "ms_per_step": round(1e3 * total_s / done, 3)}


# ---------------------------------------------------------------------------------------------

def dist_setup(args):
    """One process per GPU; NCCL for the barrier, the max-over-ranks timing and validation.
    The reference arm runs on rank 0 alone and needs no process group."""
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args, world, rank) -> int:
    """The reference arm: the reference's CPU path over the workload's full token count (the
    same configuration as the GPU arm), on rank 0 with every host thread."""
    cfg, _, pos_spec = WORKLOADS[args.workload]
    total = workload_total(args.workload, args.tokens)
    if rank != 0:
        return 0
    tokens = min(args.reference_tokens, total) if args.reference_tokens else total
    # untimed warm-up passes on a small slice, then exactly `steps` timed passes
    cpu_chain_sample(min(tokens, 4096), cfg, pos_spec, max(1, args.warmup))
    base = cpu_chain_sample(tokens, cfg, pos_spec, args.steps)
    line = {
        "metric": METRIC, "value": base["value"], "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{cfg['name']} layer-op chain, {args.workload}", "tokens": total,
                   "sample_tokens": tokens, "ops": op_names(cfg)},
        "tokens_per_s": base["tokens_per_s"], "ops_gbs": base["ops_gbs"],
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_sampling(args) -> int:
    """Greedy sampling after the LM head: argmax over bf16 logits, one op, on one GPU."""
    import torch

    import svllm_ops

    vocab = QWEN3["vocab"]
    rows = args.tokens or 1024  # 1024 x 151936 bf16 = 311 MB, above the L2
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    logits = torch.empty(rows, vocab, device=dev, dtype=torch.bfloat16).normal_(generator=g)
    for _ in range(args.warmup):
        svllm_ops.argmax(logits)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        ids = svllm_ops.argmax(logits)
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    assert torch.equal(ids, torch.argmax(logits, dim=-1))
    # the same launches replayed from a CUDA graph: the kernel's own time, without the host's
    # per-call overhead (which bounds the eager loop for small batches)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(args.steps):
            gids = svllm_ops.argmax(logits)
    graph.replay()
    torch.cuda.synchronize()
    start.record()
    graph.replay()
    stop.record()
    torch.cuda.synchronize()
    graph_ms = start.elapsed_time(stop) / args.steps
    assert torch.equal(gids, ids)
    eager_ms, ms = ms, graph_ms
    nbytes = rows * vocab * 2 + rows * 8
    peak = float(measured_peaks()["hbm_gbs"])
    print(json.dumps({
        "metric": "greedy sampling (argmax over logits) achieved HBM GB/s", "value":
        round(nbytes / (ms * 1e-3) / 1e9, 1), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "argmax over LM-head logits", "rows": rows, "vocab": vocab,
                   "l2": "no flush" if rows * vocab * 2 > 126e6 else "L2-resident"},
        "frac_of_peak": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
        "timing": "CUDA graph replay of the steps", "eager_ms_per_step": round(eager_ms, 4),
        "gpu_launches": args.steps}), flush=True)
    return 0


def run_lm_head(args) -> int:
    """The tied LM head fused with greedy sampling (svllm_ops.greedy_sample on CUDA: one tcgen05
    GEMM whose epilogue takes the argmax) against torch.matmul + svllm_ops.argmax, at the
    Qwen3-0.6B and Llama-3.2-1B vocabularies, decode to prefill batch sizes."""
    import torch

    import svllm_ops

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    peaks = measured_peaks()
    batches = [int(b) for b in args.batches.split(",")]

    def replay_us(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        stop.record()
        torch.cuda.synchronize()
        return start.elapsed_time(stop) / args.steps * 1e3

    for cfg in (QWEN3, LLAMA):
        v, h = cfg["vocab"], cfg["hidden"]
        w = (torch.randn(v, h, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        for b in batches:
            x = torch.randn(b, h, device=dev, generator=g).to(torch.bfloat16)
            fused = replay_us(lambda: svllm_ops.greedy_sample(x, w))
            split = replay_us(lambda: svllm_ops.argmax(torch.matmul(x, w.t())))
            ids = svllm_ops.greedy_sample(x, w)
            ref = torch.argmax(torch.matmul(x, w.t()), dim=-1)
            weight_bytes = v * h * 2
            flops = 2 * b * v * h
            print(json.dumps({
                "metric": "LM head + greedy sampling (fused tcgen05 GEMM + argmax)",
                "value": round(fused, 2), "unit": "us", "n_gpus": 1, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(fused / 1e3, 5),
                "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "tied LM head + argmax", "model": cfg["name"],
                           "batch": b, "vocab": v, "hidden": h,
                           "timing": "CUDA graph replay of the steps"},
                "matmul_then_argmax_us": round(split, 2), "speedup": round(split / fused, 3),
                "weight_stream_gbs": round(weight_bytes / (fused * 1e-6) / 1e9, 1),
                "weight_stream_frac_of_peak": round(weight_bytes / (fused * 1e-6) / 1e9
                                                    / float(peaks["hbm_gbs"]), 4),
                "tflops": round(flops / (fused * 1e-6) / 1e12, 1),
                "tflops_frac_of_peak": round(flops / (fused * 1e-6) / 1e12
                                             / float(peaks.get("bf16_tflops", 1590.0)), 4),
                "ids_equal_to_matmul_argmax": round(float((ids == ref).float().mean()), 6),
                "gpu_launches": 2 * args.steps}), flush=True)
    return 0


def model_weights(cfg: dict, layers: int, device, seed: int = 1234) -> dict:
    """Random Hugging Face-named weights of a Qwen3 model: projections N(0, 0.02), norm weights
    1 + N(0, 0.1), tied embedding."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    h, hq, hk, d, i, v = (cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"],
                          cfg["inter"], cfg["vocab"])

    def proj(*shape):
        return (torch.randn(*shape, device=device, generator=g) * 0.02).to(torch.bfloat16)

    def norm(n):
        return (1 + 0.1 * torch.randn(n, device=device, generator=g)).to(torch.bfloat16)

    w = {"model.embed_tokens.weight": proj(v, h), "model.norm.weight": norm(h)}
    for layer in range(layers):
        p = f"model.layers.{layer}."
        w.update({p + "input_layernorm.weight": norm(h),
                  p + "post_attention_layernorm.weight": norm(h),
                  p + "self_attn.q_proj.weight": proj(hq * d, h),
                  p + "self_attn.k_proj.weight": proj(hk * d, h),
                  p + "self_attn.v_proj.weight": proj(hk * d, h),
                  p + "self_attn.o_proj.weight": proj(h, hq * d),
                  p + "self_attn.q_norm.weight": norm(d),
                  p + "self_attn.k_norm.weight": norm(d),
                  p + "mlp.gate_proj.weight": proj(i, h),
                  p + "mlp.up_proj.weight": proj(i, h),
                  p + "mlp.down_proj.weight": proj(h, i)})
    return w


def run_model_decode(args) -> int:
    """Decode steps of Qwen3-0.6B (28 layers, random weights) through svllm_ops.Model: the fused
    ops around torch GEMMs and a LibTorch attention over a paged KV cache of `--context` random
    tokens per request, greedy sampling included; eager and replayed from CUDA graphs."""
    import torch

    import svllm_ops

    cfg, layers, block = QWEN3, 28, 16
    dev = torch.device("cuda", 0)
    batches = [int(b) for b in args.batches.split(",")]
    blocks_per_seq = -(-args.context // block)
    model = svllm_ops.Model(svllm_ops.ModelConfig(
        vocab_size=cfg["vocab"], hidden_size=cfg["hidden"], intermediate_size=cfg["inter"],
        num_layers=layers, num_heads=cfg["heads"], num_kv_heads=cfg["kv_heads"],
        head_dim=cfg["head_dim"], rms_norm_eps=cfg["eps"], rope_theta=cfg["theta"],
        tie_word_embeddings=True, qk_norm=True), model_weights(cfg, layers, dev))
    model.allocate_kv_cache(max(batches) * blocks_per_seq, block)
    g = torch.Generator(device=dev).manual_seed(3)
    for k, v in zip(model.k_cache, model.v_cache):
        k.normal_(generator=g)
        v.normal_(generator=g)
    graphs = svllm_ops.DecodeGraphs(model, max_num_seqs=max(batches),
                                    max_blocks_per_seq=blocks_per_seq, batch_sizes=batches)
    for b in batches:
        tables = torch.arange(b * blocks_per_seq, device=dev, dtype=torch.int32).view(b, -1)
        seq_lens = torch.full((b,), args.context, device=dev, dtype=torch.int32)
        pos = seq_lens.long() - 1
        slots = tables[:, -1].long() * block + pos % block
        ids = torch.randint(0, cfg["vocab"], (b,), device=dev, generator=g)
        step = dict(ids=ids, positions=pos, slot_mapping=slots, block_tables=tables,
                    seq_lens=seq_lens)
        times = {}
        for mode, fn in (("eager", model.decode), ("graph", graphs.step)):
            for _ in range(args.warmup):
                out = fn(**step)
            torch.cuda.synchronize()
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(args.steps):
                out = fn(**step)
            stop.record()
            torch.cuda.synchronize()
            times[mode] = start.elapsed_time(stop) / args.steps
            if mode == "eager":
                eager_out = out
        assert torch.equal(out, eager_out)
        print(json.dumps({
            "metric": "Qwen3-0.6B decode throughput (tokens/s)",
            "value": round(b / (times["graph"] * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(times["graph"], 4), "eager_ms_per_step": round(times["eager"], 4),
            "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (random weights, random KV cache)",
            "config": {"workload": "decode step through the model forward (28 layers, greedy)",
                       "batch": b, "context": args.context, "block_size": block,
                       "timing": "CUDA graph replay; eager alongside"}}), flush=True)
    del graphs
    return 0


def run_decode_attention(args) -> int:
    """Paged decode attention of one Qwen3-0.6B layer (16 query heads over 8 KV heads of 128,
    block size 16) at each `--batches` size with `--context` cached tokens per request, through
    the C ABI (svllm_paged_decode_attention_bf16), beside the composite it replaces in the model
    forward: gather each request's K/V pages, then torch SDPA. The block tables are a random
    permutation of the cache's blocks, so the pages a request reads are scattered."""
    import torch
    import torch.nn.functional as F

    import svllm_capi as capi

    cfg, block = QWEN3, 16
    hq, hk, d = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    peaks = measured_peaks()
    scale = d ** -0.5

    def replay_us(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        stop.record()
        torch.cuda.synchronize()
        return start.elapsed_time(stop) / args.steps * 1e3

    for b in [int(x) for x in args.batches.split(",")]:
        per_seq = -(-args.context // block)
        blocks = b * per_seq
        k_cache = torch.randn(blocks, block, hk, d, device=dev, generator=g).to(torch.bfloat16)
        v_cache = torch.randn(blocks, block, hk, d, device=dev, generator=g).to(torch.bfloat16)
        tables = torch.randperm(blocks, device=dev, generator=g).view(b, per_seq).int()
        seq_lens = torch.full((b,), args.context, device=dev, dtype=torch.int32)
        q = torch.randn(b, hq, d, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty_like(q)
        max_len = per_seq * block

        def kernel():
            capi.paged_decode_attention(out, q, k_cache, v_cache, tables, seq_lens, max_len,
                                        scale)

        slots = (tables.long()[:, :, None] * block
                 + torch.arange(block, device=dev)).view(b, -1)[:, :args.context]

        def composite():
            k = k_cache.view(-1, hk, d).index_select(0, slots.reshape(-1)).view(b, -1, hk, d)
            v = v_cache.view(-1, hk, d).index_select(0, slots.reshape(-1)).view(b, -1, hk, d)
            return F.scaled_dot_product_attention(q[:, :, None], k.transpose(1, 2),
                                                  v.transpose(1, 2), scale=scale,
                                                  enable_gqa=True)[:, :, 0]

        us = replay_us(kernel)
        ref_us = replay_us(composite)
        kernel()
        ref = composite().float()
        err = float((out.float() - ref).abs().max())
        # algorithmic bytes: the K and V rows each request reads, q, out, its table row and length
        traffic = (2 * b * args.context * hk * d * 2 + 2 * b * hq * d * 2 + b * per_seq * 4
                   + b * 4)
        gbs = traffic / (us * 1e-6) / 1e9
        print(json.dumps({
            "metric": "paged decode attention (KV bytes streamed per second)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5), "us_per_launch": round(us, 2),
            "higher_is_better": True, "dtype": "bf16 (fp32 softmax and accumulation)",
            "data": "synthetic (random q and KV cache, scattered pages)",
            "config": {"workload": "Qwen3-0.6B layer decode attention", "batch": b,
                       "context": args.context, "heads": hq, "kv_heads": hk, "head_dim": d,
                       "block_size": block, "kv_bytes": 2 * b * args.context * hk * d * 2,
                       "timing": "CUDA graph replay of the steps"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1),
                         "peak": float(peaks["hbm_gbs"]),
                         "unit": "GB/s", "frac": round(gbs / float(peaks["hbm_gbs"]), 4)},
            "gather_then_sdpa_us": round(ref_us, 2), "speedup": round(ref_us / us, 3),
            "max_abs_err_vs_sdpa": round(err, 6),
            "gpu_launches": args.steps}), flush=True)
        del k_cache, v_cache
    return 0


def run_decode_linear(args) -> int:
    """The four projections of a Qwen3-0.6B layer (qkv, o, gate_up, down) at each `--batches`
    size up to 16 rows, through the C ABI (svllm_decode_linear_bf16), beside torch.matmul
    (cuBLAS) on the same operands. At these sizes the work is a stream over the weight: the
    roofline is HBM bandwidth on the weight bytes (plus the activations in and out)."""
    import torch

    import svllm_capi as capi

    cfg = QWEN3
    h, d = cfg["hidden"], cfg["head_dim"]
    shapes = {"qkv": ((cfg["heads"] + 2 * cfg["kv_heads"]) * d, h),
              "o_proj": (h, cfg["heads"] * d), "gate_up": (2 * cfg["inter"], h),
              "down": (h, cfg["inter"])}
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(17)
    peaks = measured_peaks()

    def replay_us(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        stop.record()
        torch.cuda.synchronize()
        return start.elapsed_time(stop) / args.steps * 1e3

    # one weight per step of the replay, so that consecutive launches do not find it in L2
    copies = max(2, -(-256 * 2 ** 20 // min(n * k * 2 for n, k in shapes.values())))
    for name, (n, k) in shapes.items():
        ws = [(torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
              for _ in range(copies)]
        for b in [int(x) for x in args.batches.split(",") if int(x) <= 16]:
            x = torch.randn(b, k, device=dev, generator=g).to(torch.bfloat16)
            out = torch.empty(b, n, device=dev, dtype=torch.bfloat16)
            it = {"i": 0}

            def ours():
                capi.decode_linear(out, x, ws[it["i"] % copies])
                it["i"] += 1

            def cublas():
                torch.matmul(x, ws[it["i"] % copies].t())
                it["i"] += 1

            us = replay_us(ours)
            ref_us = replay_us(cublas)
            capi.decode_linear(out, x, ws[0])
            err = float((out.float() - (x.float() @ ws[0].float().t())).abs().max())
            traffic = n * k * 2 + b * k * 2 + b * n * 2
            gbs = traffic / (us * 1e-6) / 1e9
            print(json.dumps({
                "metric": "decode linear (weight bytes streamed per second)",
                "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5),
                "us_per_launch": round(us, 2), "higher_is_better": True,
                "dtype": "bf16 (fp32 accumulation)", "data": "synthetic",
                "config": {"workload": f"Qwen3-0.6B {name} projection", "rows": b,
                           "out_features": n, "in_features": k, "weight_copies": copies,
                           "timing": "CUDA graph replay, a different weight copy per launch "
                                     "(the copies exceed L2)"},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1),
                             "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                             "frac": round(gbs / float(peaks["hbm_gbs"]), 4)},
                "cublas_us": round(ref_us, 2), "speedup": round(ref_us / us, 3),
                "max_abs_err_vs_fp32": round(err, 6), "gpu_launches": args.steps}),
                flush=True)
        del ws
    return 0


# ---------------------------------------------------------------------------------------------
# The benchmark definition's other configurations, measured in the same run at N=1 (rank 0):
# config 0 fp32 (GPU through the C ABI's fp32 entry points, CPU through the fp32 restatement),
# config 1 decode, config 2 packed prefill, config 3 Llama (factors 32 and 8). Each chain pass is
# replayed from a CUDA graph: at these sizes the host's per-launch cost would otherwise be timed.

class CapiChain:
    """The chain through the C ABI (svllm_capi): used for fp32, which svllm_ops (bf16 only, like
    the reference's op API) does not take."""

    def __init__(self, inp: dict, cfg: dict):
        import torch
        import svllm_ops

        self.inp, self.cfg = inp, cfg
        T, dt = inp["ids"].shape[0], inp["x"].dtype
        dev = inp["ids"].device
        self.emb_out = torch.empty(T, cfg["hidden"], device=dev, dtype=dt)
        self.silu_out = torch.empty(T, cfg["inter"], device=dev, dtype=dt)
        self.inv = svllm_ops.rope_inv_freq(cfg["theta"], cfg["head_dim"], scaling_of(cfg)).tolist()

    def run_op(self, name: str) -> None:
        import svllm_capi as capi

        i, c = self.inp, self.cfg
        if name == "embedding":
            capi.embedding(self.emb_out, i["ids"], i["table"])
        elif name == "add_rms_norm":
            capi.add_rms_norm(i["x"], i["residual"], i["w"], c["eps"])
        elif name == "qk_norm_rope":
            capi.qk_norm_rope(i["q"], i["k"], i["qw"], i["kw"], i["pos"], c["eps"], self.inv)
        elif name == "rope":
            capi.rope(i["q"], i["k"], i["pos"], self.inv)
        else:
            capi.silu_and_mul(self.silu_out, i["gate"], i["up"])


def graph_chain_us(chain, names: list[str], reps: int, warmup: int) -> float:
    """Microseconds per pass of the chain, `reps` passes captured in one CUDA graph and the
    graph replayed (after `warmup` eager passes and one untimed replay)."""
    import torch

    for _ in range(max(1, warmup)):
        for op in names:
            chain.run_op(op)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    capture = torch.cuda.Stream()
    capture.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(capture):
        with torch.cuda.graph(graph, stream=capture):
            for _ in range(reps):
                for op in names:
                    chain.run_op(op)
    torch.cuda.current_stream().wait_stream(capture)
    graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replays = 3
    start.record()
    for _ in range(replays):
        graph.replay()
    stop.record()
    torch.cuda.synchronize()
    del graph
    return start.elapsed_time(stop) * 1e3 / (replays * reps)


def cpu_fp32_chain(tokens: int, cfg: dict, pos_hi: int, steps: int) -> dict:
    """Config 0's CPU side: the fp32 chain through the C/OpenMP restatement (the reference has
    no fp32 kernel: its op API rejects fp32) with every host thread."""
    import numpy as np

    import oracle

    cores = len(os.sched_getaffinity(0))
    threads = oracle.set_num_threads(cores)
    rng = np.random.default_rng(99)
    h, hd, inter = cfg["hidden"], cfg["head_dim"], cfg["inter"]

    def f32(*shape, scale=1.0, shift=0.0):
        return (rng.standard_normal(shape, dtype=np.float32) * scale + shift).astype(np.float32)

    table = f32(cfg["vocab"], h, scale=0.02)
    ids = rng.integers(0, cfg["vocab"], tokens, dtype=np.int32)
    x, r, w = f32(tokens, h), f32(tokens, h), f32(h, scale=0.1, shift=1.0)
    q, k = f32(tokens, cfg["heads"], hd), f32(tokens, cfg["kv_heads"], hd)
    qw, kw = f32(hd, scale=0.1, shift=1.0), f32(hd, scale=0.1, shift=1.0)
    pos = rng.integers(0, pos_hi, tokens, dtype=np.int64)
    gate, up = f32(tokens, inter), f32(tokens, inter)
    emb_out, silu_out = np.empty((tokens, h), np.float32), np.empty((tokens, inter), np.float32)
    inv = oracle.inv_freq(cfg["theta"], hd, cfg["scaling"])

    def chain():
        oracle.embedding(ids, table, out=emb_out)
        oracle.add_rms_norm(x, r, w, cfg["eps"], inplace=True)
        oracle.qk_norm_rope(q, k, qw, kw, pos, cfg["eps"], inv, inplace=True)
        oracle.silu_and_mul(gate, up, out=silu_out)

    chain()
    t0 = time.perf_counter()
    for _ in range(steps):
        chain()
    sec = (time.perf_counter() - t0) / steps
    nbytes = sum(op_bytes(cfg, elem=4).values()) * tokens
    return {"value": round(nbytes / sec / 1e9, 2), "unit": UNIT, "cores": cores, "kind": "port",
            "us_per_chain": round(sec * 1e6, 1),
            "sample": f"{tokens} tokens x {steps} passes of the fp32 chain on host memory, "
                      f"{threads} OpenMP threads; C/OpenMP restatement (oracle/): the reference "
                      "rejects fp32"}


def measure_configs(args, dev, peak: float) -> dict:
    """Configs 0-3 of the benchmark definition at their own sizes, one CUDA-graph timing each,
    with the SM clock sampled around it."""
    import torch

    out = {}
    cases = [
        ("config0_fp32", "decode", dict(QWEN3), torch.float32),
        ("config1_decode", "decode", dict(QWEN3), torch.bfloat16),
        ("config2_prefill", "prefill", dict(QWEN3), torch.bfloat16),
        ("config3_llama_factor32", "llama", dict(LLAMA), torch.bfloat16),
        ("config3_llama_factor8", "llama", dict(LLAMA, scaling=(8.0, 1.0, 4.0, 8192)),
         torch.bfloat16),
    ]
    for key, workload, cfg, dtype in cases:
        _, _, pos_spec = WORKLOADS[workload]
        if key == "config0_fp32":
            pos_spec = ("packed", 256)  # positions 0..255
        T = workload_total(workload)
        inp = make_inputs(T, pos_spec, cfg, dev, seed=4242)
        if dtype == torch.float32:
            inp = {k: (v.float() if v.dtype == torch.bfloat16 else v) for k, v in inp.items()}
            chain = CapiChain(inp, cfg)
        else:
            chain = Chain(inp, cfg)
        names = op_names(cfg)
        reps = 20 if T <= 4096 else 2
        sampler = ClockSampler([dev.index])
        with sampler:
            us = graph_chain_us(chain, names, reps, args.warmup)
        nbytes = sum(op_bytes(cfg, elem=4 if dtype == torch.float32 else 2).values()) * T
        gbs = nbytes / (us * 1e-6) / 1e9
        entry = {
            "tokens": T, "dtype": "f32" if dtype == torch.float32 else "bf16",
            "positions": positions_label(pos_spec), "ops": names,
            "rope_scaling": cfg["scaling"], "us_per_chain": round(us, 2),
            "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4),
            "tokens_per_s": round(T / (us * 1e-6), 1), "cuda_graph": True,
            "l2": ("inputs L2-resident (decode-sized; not flushed)" if nbytes < 126e6 else
                   "each pass streams more than the 126 MB L2"),
            "clocks": sampler.summary(),
        }
        if key == "config0_fp32" and not args.no_cpu_baseline:
            entry["cpu_baseline"] = cpu_fp32_chain(T, cfg, 4096, max(20, args.steps))
        out[key] = entry
        del chain, inp
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------
# RMSNorm alone, the one op the reference ships a CUDA kernel for: svllm_ops.rms_norm (--impl
# ours) or the reference's own op API on its own CUDA kernel, built from its sources into
# oracle/_ref (--impl reference), timed the same way on the same shapes.

RMS_SHAPES = [(1_048_576, 1024), (16_384, 2048), (1_048_576 * 16, 128)]


def run_rms_norm(args) -> int:
    import torch

    dev = torch.device("cuda", 0)
    if args.impl == "reference":
        import oracle

        op = oracle.reference_module()
        if op is None:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference's rms_norm was not built into oracle/_ref"}))
            return 0
        fn, label = op.rms_norm, "reference CUDA rms_norm (its src/ops/cuda/rms_norm.cu, sm_100a)"
    else:
        import svllm_ops

        fn, label = svllm_ops.rms_norm, "svllm_ops.rms_norm (sm_100a bulk-copy kernel)"
    g = torch.Generator(device=dev).manual_seed(17)
    peak = float(measured_peaks()["hbm_gbs"])
    shapes = {}
    # --tokens N: one shape, N rows of 1024 (a small case for a profiler)
    run_shapes = [(args.tokens, 1024)] if args.tokens else RMS_SHAPES
    sampler = ClockSampler([0])
    with sampler:
        for rows, hidden in run_shapes:
            x = torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16).normal_(generator=g)
            w = (torch.empty(hidden, device=dev).normal_(generator=g) * 0.1 + 1).to(torch.bfloat16)
            for _ in range(args.warmup):
                fn(x, w, 1e-6)
            torch.cuda.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(args.steps):
                fn(x, w, 1e-6)
            stop.record()
            torch.cuda.synchronize()
            ms = start.elapsed_time(stop) / args.steps
            nbytes = rows * hidden * 4  # read x, write out (bf16); the weight is amortised
            shapes[f"{rows}x{hidden}"] = {"ms": round(ms, 4),
                                          "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                                          "frac_of_peak": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)}
            del x
            torch.cuda.empty_cache()
    head = shapes[f"{run_shapes[0][0]}x{run_shapes[0][1]}"]
    line = {"metric": "rms_norm achieved HBM GB/s", "value": head["gbs"], "unit": UNIT,
            "impl": args.impl, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms"], "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "rms_norm, bf16, x ~ N(0,1), weight 1+N(0,0.1), eps 1e-6",
                       "shapes": [f"{r}x{h}" for r, h in run_shapes],
                       "timing": "CUDA events around `steps` back-to-back calls of the op API "
                                 "(output allocation included, as the API allocates it)",
                       "l2": "inputs larger than L2 except 16384x2048 (67 MB: L2-warm)"},
            "op": label, "shapes": shapes, "peak": peak, "clocks": sampler.summary()}
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    args = parse_args()
    if args.workload == "sampling":
        return run_sampling(args)
    if args.workload == "model-decode":
        return run_model_decode(args)
    if args.workload == "lm-head":
        return run_lm_head(args)
    if args.workload == "decode-attention":
        return run_decode_attention(args)
    if args.workload == "decode-linear":
        return run_decode_linear(args)
    if args.workload == "rms-norm":
        return run_rms_norm(args)
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    import torch.distributed as dist

    import svllm_ops

    assert torch.cuda.is_available(), "bench.py (impl ours) needs a GPU"
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg, _, pos_spec = WORKLOADS[args.workload]
    total = workload_total(args.workload, args.tokens)
    if args.kv_cache:
        # the cache variant is measured on the device; e2e, the CPU leg and validation cover the
        # headline chain
        cfg = dict(cfg, kv_cache=True)
        args.no_e2e = args.no_cpu_baseline = args.no_validate = True
    names = op_names(cfg)
    begin, end = split_rows(total, world, rank)
    T = end - begin
    nbytes = op_bytes(cfg)
    chain_bytes_per_token = sum(nbytes.values())

    inp = make_inputs(T, pos_spec, cfg, dev, seed=1000 + rank, first_row=begin)
    chain = Chain(inp, cfg)
    torch.cuda.synchronize()

    validation = None
    if not args.no_validate:
        validation = validate(chain, inp, cfg, world, rank, dev)

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        for op in names:
            chain.run_op(op)
    torch.cuda.synchronize()
    assert svllm_ops.read_device_error(local, True) == 0

    ev = {op: [] for op in names}
    graph = None
    if args.graph:
        # one graph holds the whole chain: the launch latency of four kernels becomes one replay
        graph = torch.cuda.CUDAGraph()
        capture = torch.cuda.Stream()
        capture.wait_stream(stream)
        with torch.cuda.stream(capture):
            with torch.cuda.graph(graph, stream=capture):
                for op in names:
                    chain.run_op(op)
        stream.wait_stream(capture)
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
    sampler = ClockSampler(list(range(world)) if world > 1 else [local], enabled=rank == 0)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                for op in names:
                    chain.run_op(op)
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = start.elapsed_time(stop)
    # Per-op times come from a second pass of the same steps with events around each launch
    # (outside the timed region: events between kernels would stand in the way of the next
    # kernel's early launch, and a graph replay has no per-op events).
    for _ in range(args.steps):
        for op in names:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            chain.run_op(op)
            e1.record(stream)
            ev[op].append((e0, e1))
    torch.cuda.synchronize()
    if graph is not None:
        del graph
    op_ms = {op: sum(a.elapsed_time(b) for a, b in ev[op]) / args.steps for op in names}
    op_ms_median = {op: statistics.median(a.elapsed_time(b) for a, b in ev[op]) for op in names}
    # ids repeat (T / V ~ 6.9 at 1M tokens), so the L2 can serve repeated table rows: the bytes
    # of the distinct rows read, beside the algorithmic bytes, keep the embedding figure honest
    unique_rows = int(torch.unique(inp["ids"]).numel()) if "embedding" in names else 0

    t = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item()) / args.steps  # per step, slowest rank

    # end to end through svllm_ops with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(chain, inp, cfg, args, world, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_chain_sample(min(args.cpu_sample_tokens, total), cfg, pos_spec, 2,
                               min_seconds=10.0)

    configs = None
    if rank == 0 and world == 1 and args.workload == "sweep" and not args.no_configs:
        configs = measure_configs(args, dev, float(measured_peaks()["hbm_gbs"]))

    if rank == 0:
        peaks = measured_peaks()
        peak = float(peaks["hbm_gbs"])
        value = chain_bytes_per_token * total / (max_ms * 1e-3) / 1e9
        ops_gbs = {op: round(nbytes[op] * T / (op_ms[op] * 1e-3) / 1e9, 1) for op in names}
        dominant = max(names, key=lambda op: op_ms[op])
        traffic = load_traffic(dominant, T)
        achieved = nbytes[dominant] * T / (op_ms[dominant] * 1e-3) / 1e9
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(max_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{cfg['name']} layer-op chain, {args.workload}",
                       "tokens": total, "tokens_per_gpu": T, "hidden": cfg["hidden"],
                       "heads": [cfg["heads"], cfg["kv_heads"]], "head_dim": cfg["head_dim"],
                       "intermediate": cfg["inter"], "vocab": cfg["vocab"],
                       "positions": positions_label(pos_spec),
                       "rope_scaling": cfg["scaling"], "ops": names,
                       "l2": "no flush: every op's inputs exceed the 126 MB L2"
                       if T * 2 * cfg["hidden"] > 126e6 else "inputs L2-resident (small T)",
                       "parallelism": f"rows sharded over {world} GPU(s), no collective"},
            "tokens_per_s": round(total / (max_ms * 1e-3), 1),
            "frac_of_peak": round(value / (peak * world), 4),
            "ops_gbs_per_gpu": ops_gbs,
            "ops_ms_per_gpu": {op: round(op_ms[op], 4) for op in names},
            "ops_ms_median_per_gpu": {op: round(op_ms_median[op], 4) for op in names},
            "frac_of_nominal": round(value / (NOMINAL_HBM_GBS * world), 4),
            "embedding_unique_rows": {
                "rows": unique_rows, "of_tokens": T,
                "gbs": round((unique_rows * 2 * cfg["hidden"] + T * (2 * cfg["hidden"] + 4))
                             / (op_ms["embedding"] * 1e-3) / 1e9, 1)}
            if "embedding" in names else None,
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic,
                         "algorithmic_bytes": nbytes[dominant] * T,
                         "kernel_timing": "CUDA events around each launch, on the launching "
                                          "stream, in a second pass of the same K steps",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"
                         if not peaks.get("fallback") else "fallback 6650 GB/s"},
            "clocks": clocks,
            "gpu_launches": len(names) * args.steps,
            "cuda_graph": bool(args.graph),
            "e2e": e2e,
            "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
            if cpu else None,
            "validation": validation,
            "configs": configs,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def load_traffic(kernel_op: str, tokens: int):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, scaled to
    this launch's tokens (traffic grows with the rows processed); None if there is none."""
    path = ROOT / "profiles" / "dram_traffic.json"
    if not path.exists():
        return None
    data = json.loads(path.read_text())
    entry = data.get(kernel_op)
    if not entry:
        return None
    return round(entry["bytes_per_token"] * tokens)


# ---------------------------------------------------------------------------------------------
# Validation (outside every timed region), against two references:
#   * the same GPU's torch composites of the formulas, on every rank: index_select for the
#     gather, a bf16 add for the residual, the reference test's own RMSNorm composite
#     (tests/python/test_rms_norm.py:24-27: F.rms_norm in fp32, rounded, times the weight) for the
#     norms, Hugging Face's rotary embedding, F.silu(gate) * up. The gather, the residual and
#     SiLU * up must agree bit for bit; the norms differ from the composite only in summation
#     order (the kernels replay the reference CUDA kernel's), so those outputs are held to 2 bf16
#     ulp or 2^-7 of the row's largest magnitude, and their max-abs error is reported;
#   * svllm_ops' CPU backend on rank 0, after an NCCL all-gather of every rank's first rows
#     (the one collective of the sharded run), under the same bars (the CPU's cosf/sinf/expf are
#     the C library's, not CUDA's).

def _compare(got, want, exact: bool) -> dict:
    import numpy as np
    import torch

    def bits(t):
        return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16).astype(np.int32)

    a, b = bits(got), bits(want)
    ulp = np.abs(np.where(a & 0x8000, -(a & 0x7FFF), a) - np.where(b & 0x8000, -(b & 0x7FFF), b))
    av, bv = got.float().cpu().numpy(), want.float().cpu().numpy()
    flat_b = np.abs(bv).reshape(bv.shape[0], -1).max(axis=1)
    tol = (2.0 ** -7 * flat_b).reshape((-1,) + (1,) * (bv.ndim - 1))
    within = (ulp <= 2) | (np.abs(av - bv) <= tol)
    good = bool((ulp == 0).all()) if exact else bool(within.all())
    scale = np.maximum(flat_b, np.finfo(np.float32).tiny).reshape(tol.shape)
    return {"worst_bf16_ulp": int(ulp.max()), "not_bit_exact": int((ulp > 0).sum()),
            "max_abs": float(np.abs(av - bv).max()),
            "worst_abs_err_over_row_max": float((np.abs(av - bv) / scale).max()),
            "bit_exact_required": exact, "ok": good}


def torch_composites(saved: dict, inp: dict, cfg: dict) -> dict:
    """The chain's outputs for the saved inputs, by torch ops on the inputs' device."""
    import torch
    import torch.nn.functional as F

    import svllm_ops

    eps, d = cfg["eps"], cfg["head_dim"]
    bf = torch.bfloat16

    def norm(x, w):
        return F.rms_norm(x.float(), (x.shape[-1],), eps=eps).to(bf) * w

    inv = svllm_ops.rope_inv_freq(cfg["theta"], d, scaling_of(cfg)).to(saved["q"].device)

    def rope(x, pos):
        freqs = pos.float()[:, None] * inv[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos().to(bf)[:, None, :], emb.sin().to(bf)[:, None, :]
        half = x.shape[-1] // 2
        return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin

    r = saved["x"] + saved["residual"]
    q, k = saved["q"], saved["k"]
    if cfg["qk_norm"]:
        q, k = norm(q, inp["qw"]), norm(k, inp["kw"])
    return {"embedding": inp["table"].index_select(0, saved["ids"].long()),
            "x": norm(r, inp["w"]), "residual": r,
            "q": rope(q, saved["pos"]), "k": rope(k, saved["pos"]),
            "silu": F.silu(saved["gate"]) * saved["up"]}


EXACT_OUTPUTS = ("embedding", "residual", "silu")


def validate(chain, inp, cfg, world, rank, dev, rows: int = 256):
    import torch
    import torch.distributed as dist

    import svllm_dist
    import svllm_ops

    n = min(rows, inp["ids"].shape[0])
    if world > 1:
        t = torch.tensor([n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        n = int(t.item())
    saved = {k: inp[k][:n].clone() for k in ("ids", "x", "residual", "q", "k", "pos", "gate",
                                            "up")}
    for op in op_names(cfg):
        chain.run_op(op)
    torch.cuda.synchronize()
    got = {"embedding": chain.emb_out[:n], "x": inp["x"][:n], "residual": inp["residual"][:n],
           "q": inp["q"][:n], "k": inp["k"][:n], "silu": chain.silu_out[:n]}

    # every rank against its own GPU's torch composites; the worst over ranks is reported
    comp = torch_composites(saved, inp, cfg)
    gpu_report = {name: _compare(got[name], comp[name], name in EXACT_OUTPUTS) for name in got}
    if world > 1:
        for name, rep in gpu_report.items():
            v = torch.tensor([rep["worst_bf16_ulp"], rep["not_bit_exact"], rep["max_abs"],
                              rep["worst_abs_err_over_row_max"], 0.0 if rep["ok"] else 1.0],
                             device=dev, dtype=torch.float64)
            mx = v.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            dist.all_reduce(v, op=dist.ReduceOp.SUM)
            rep.update({"worst_bf16_ulp": int(mx[0]), "not_bit_exact": int(v[1]),
                        "max_abs": float(mx[2]), "worst_abs_err_over_row_max": float(mx[3]),
                        "ok": bool(mx[4] == 0)})

    def gather(t):
        return svllm_dist.all_gather_rows(t.contiguous(), n * world) if world > 1 else t

    got = {k: gather(v).cpu() for k, v in got.items()}
    ins = {k: gather(v).cpu() for k, v in saved.items()}
    if rank != 0:
        return None

    ops = svllm_ops
    emb = ops.embedding(ins["ids"], inp["table"].cpu())
    x, r = ins["x"].clone(), ins["residual"].clone()
    ops.add_rms_norm(x, r, inp["w"].cpu(), cfg["eps"])
    q, k = ins["q"].clone(), ins["k"].clone()
    if cfg["qk_norm"]:
        ops.qk_norm_rope(q, k, inp["qw"].cpu(), inp["kw"].cpu(), ins["pos"], cfg["eps"],
                         cfg["theta"], scaling_of(cfg))
    else:
        ops.rope(q, k, ins["pos"], cfg["theta"], scaling_of(cfg))
    y = ops.silu_and_mul(ins["gate"], ins["up"])
    want = {"embedding": emb, "x": x, "residual": r, "q": q, "k": k, "silu": y}
    cpu_report = {name: _compare(got[name], want[name], name in ("embedding", "residual"))
                  for name in want}
    ok = all(v["ok"] for v in gpu_report.values()) and all(v["ok"] for v in cpu_report.values())
    return {"rows_per_gpu": n, "gathered_from": world,
            "same_gpu_torch_composites": gpu_report, "cpu_backend": cpu_report, "ok": ok}


# ---------------------------------------------------------------------------------------------
# End to end: pinned host inputs -> device -> chain through svllm_ops -> pinned host outputs,
# pipelined in chunks over three streams (copy in, compute, copy out) so PCIe runs both ways
# while the kernels work. Every step copies all of that step's inputs in and outputs out.

def measure_e2e(chain, inp, cfg, args, world, dev):
    """The chain end to end through the C ABI (svllm_capi: the drop-in boundary a host program
    binds) from and to pinned host buffers: every step copies each chunk's inputs in, runs the
    four ops on the chunk (the gather and SiLU writing straight into the device buffers that are
    copied out), and copies every output back; copies and kernels overlap across chunks on
    three streams."""
    import torch
    import torch.distributed as dist

    import svllm_capi as capi
    import svllm_ops

    T = inp["ids"].shape[0]
    names_in = ["ids", "x", "residual", "q", "k", "pos", "gate", "up"]
    host_in = {k: torch.empty(inp[k].shape, dtype=inp[k].dtype, pin_memory=True)
               for k in names_in}
    for k in names_in:
        host_in[k].copy_(inp[k])
    out_shapes = {"emb": (T, cfg["hidden"]), "x": (T, cfg["hidden"]),
                  "residual": (T, cfg["hidden"]), "q": tuple(inp["q"].shape),
                  "k": tuple(inp["k"].shape), "silu": (T, cfg["inter"])}
    host_out = {k: torch.empty(s, dtype=torch.bfloat16, pin_memory=True)
                for k, s in out_shapes.items()}
    silu_dev = torch.empty(T, cfg["inter"], device=dev, dtype=torch.bfloat16)
    emb_dev = torch.empty(T, cfg["hidden"], device=dev, dtype=torch.bfloat16)
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out.values())
    inv = svllm_ops.rope_inv_freq(cfg["theta"], cfg["head_dim"], scaling_of(cfg)).tolist()

    chunks = max(1, min(16, T // 16384))
    bounds = [(T * c // chunks, T * (c + 1) // chunks) for c in range(chunks)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp = torch.cuda.current_stream(dev)

    done_out: list = [None] * len(bounds)

    def step():
        done_in, done_comp = [], []
        for c, (a, b) in enumerate(bounds):
            with torch.cuda.stream(s_in):
                if done_out[c] is not None:
                    # the previous step's copy-out of this chunk must finish before we overwrite
                    s_in.wait_event(done_out[c])
                for k in names_in:
                    inp[k][a:b].copy_(host_in[k][a:b], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                done_in.append(e)
        for c, (a, b) in enumerate(bounds):
            s_comp.wait_event(done_in[c])
            capi.embedding(emb_dev[a:b], inp["ids"][a:b], inp["table"])
            capi.add_rms_norm(inp["x"][a:b], inp["residual"][a:b], inp["w"], cfg["eps"])
            if cfg["qk_norm"]:
                capi.qk_norm_rope(inp["q"][a:b], inp["k"][a:b], inp["qw"], inp["kw"],
                                  inp["pos"][a:b], cfg["eps"], inv)
            else:
                capi.rope(inp["q"][a:b], inp["k"][a:b], inp["pos"][a:b], inv)
            capi.silu_and_mul(silu_dev[a:b], inp["gate"][a:b], inp["up"][a:b])
            e = torch.cuda.Event()
            e.record(s_comp)
            done_comp.append(e)
        for c, (a, b) in enumerate(bounds):
            with torch.cuda.stream(s_out):
                s_out.wait_event(done_comp[c])
                host_out["emb"][a:b].copy_(emb_dev[a:b], non_blocking=True)
                host_out["x"][a:b].copy_(inp["x"][a:b], non_blocking=True)
                host_out["residual"][a:b].copy_(inp["residual"][a:b], non_blocking=True)
                host_out["q"][a:b].copy_(inp["q"][a:b], non_blocking=True)
                host_out["k"][a:b].copy_(inp["k"][a:b], non_blocking=True)
                host_out["silu"][a:b].copy_(silu_dev[a:b], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_out)
                done_out[c] = e

    step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(s_comp)
    for _ in range(args.steps):
        step()
    s_comp.wait_stream(s_out)
    s_comp.wait_stream(s_in)
    stop.record(s_comp)
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    total = T * world if world > 1 else T
    if world > 1:
        tt = torch.tensor([T], device=dev, dtype=torch.int64)
        dist.all_reduce(tt)
        total = int(tt.item())
    value = sum(op_bytes(cfg).values()) * total / (ms * 1e-3) / 1e9
    # the PCIe bound with every rank copying at once, as they do in the timed steps
    bound = pcie_bound_ms(dev, h2d, d2h, world)
    return {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d * world,
            "d2h_bytes_per_step": d2h * world, "ms_per_step": round(ms, 3),
            "chunks": chunks, "api": "C ABI through svllm_capi (pinned host buffers, 3 streams)",
            "pcie": {**bound, "frac": round(bound["bound_ms"] / ms, 4)}}


def pcie_bound_ms(dev, h2d: int, d2h: int, world: int = 1) -> dict:
    """The step time PCIe alone allows: pinned-buffer copies measured here, one direction alone
    and both at once, with every rank copying at the same time (a barrier starts each
    measurement; the slowest rank's rate counts); the copy-out overlaps the copy-in at the
    two-way rate, the rest of the larger direction runs at the one-way rate."""
    import torch
    import torch.distributed as dist

    n = 1 << 29
    hs = [torch.empty(n, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    ds = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        sec = torch.tensor([(time.perf_counter() - t0) / 3], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(sec, op=dist.ReduceOp.MAX)
        return float(sec.item())

    def one_way():
        with torch.cuda.stream(s_in):
            ds[0].copy_(hs[0], non_blocking=True)

    def two_way():
        with torch.cuda.stream(s_in):
            ds[0].copy_(hs[0], non_blocking=True)
        with torch.cuda.stream(s_out):
            hs[1].copy_(ds[1], non_blocking=True)

    one = n / timed(one_way)
    both = n / timed(two_way)
    small, large = sorted((h2d, d2h))
    bound_s = small / both + (large - small) / one
    return {"one_way_gbs": round(one / 1e9, 1), "two_way_gbs_each": round(both / 1e9, 1),
            "bound_ms": round(bound_s * 1e3, 1), "ranks_copying_at_once": world}


if __name__ == "__main__":
    sys.exit(main())
