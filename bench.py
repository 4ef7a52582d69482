"""Benchmark of the D2-SD verify hot path on B200.

Headline (the north-star shape, on Qwen3-8B's 36 layers):
one verify step of one request = for every layer, the two-level cascade
attention of 8 branches x 32 block tokens over a 32768-token paged prefix
(kernel a: shared prefix on tcgen05/TMEM, kernel b: per-branch causal suffix
fused with the LSE merge), then greedy acceptance over the bf16 target logits
[8, 32, 151936] (kernel c), then the commit of the accepted rows into all 36
layers' paged caches (kernel d). Metric: verified tokens/s (B*T / step time).

The same JSON line carries the other BASELINE configs under "configs":
  cfg4  batched serving: 64 requests (prefix ~ U[512, 8192], 4 x 16 tokens),
        36 layers of attention over one page pool, batched acceptance and
        commit; request-parallel over the GPUs (LPT), no collective.
  cfg5  GPT-OSS-20B attention shapes: 24 layers alternating 128-token sliding
        window and full attention with sinks, prefix 16384, 6 x 16 tokens,
        acceptance over V 201088; KV-head sharded like config 3.
  cfg2  Qwen3-8B (random init, bf16, 36 layers) full cascade_verify_forward of
        4 x 32 candidates over a 2048-token prefix (1 GPU).
  cfg1  the fp32 single-layer case: the fp32 cascade kernel and acceptance over
        fp32 logits (1 GPU).

Multi-GPU (torchrun, one rank per GPU): KV-head sharding for configs 3 and 5
(rank r owns Hk/N kv heads and their pages; kernel (b) stores each layer's
output rows into every rank's buffer over NVLink; acceptance is vocabulary
sharded, each rank scanning V/N columns and trading the rows' bests over
NVLink inside kernel (c)); request parallelism for config 4.

--impl reference: the reference's CPU path (torch.sdpa tree-masked attention +
the acceptance walk + the cat-based commit, restated in oracle/) on the host
cores, one whole layer per sample, extrapolated over the layers.
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
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

CFG3 = dict(layers=36, prefix=32768, branches=8, block=32, qo_heads=32, kv_heads=8, head_dim=128,
            vocab=151936, page_size=16, shared=0)
CFG4 = dict(layers=36, requests=64, prefix_lo=512, prefix_hi=8192, branches=4, block=16,
            qo_heads=32, kv_heads=8, head_dim=128, vocab=151936, seed=4)
CFG5 = dict(layers=24, window=128, prefix=16384, branches=6, block=16, qo_heads=64, kv_heads=8,
            head_dim=64, vocab=201088)
CFG2 = dict(layers=36, hidden=4096, intermediate=12288, qo_heads=32, kv_heads=8, head_dim=128,
            vocab=151936, prefix=2048, branches=4, block=32, rope_theta=1e6)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["d2sd", "reference"], default="d2sd")
    ap.add_argument("--configs", default="3,4,5,2,1",
                    help="configs to run; 3 is the headline line, the others go under 'configs'")
    ap.add_argument("--layers", type=int, default=CFG3["layers"])
    ap.add_argument("--prefix", type=int, default=CFG3["prefix"])
    ap.add_argument("--branches", type=int, default=CFG3["branches"])
    ap.add_argument("--block", type=int, default=CFG3["block"])
    ap.add_argument("--shared", type=int, default=CFG3["shared"],
                    help="tokens every branch shares (tree trunk); 0 = independent branches")
    ap.add_argument("--kv-layout", choices=["umma", "hnd"], default="umma",
                    help="page format of the target cache (tensor-core order or plain rows)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="multi-GPU output all-gather: kernel (b)'s own NVLink stores, or NCCL")
    ap.add_argument("--sub-layers", type=int, default=0,
                    help="layers of configs 4 and 5 (0 = their own: 36 and 24); smaller cases "
                         "for profiling")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--flashinfer", action="store_true",
                    help="config 3, one GPU: also time the reference's own GPU path (FlashInfer "
                         "kernels, JIT-compiled on first use) on the same inputs and compare")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks sampled during the timed region, peaks, profile figures
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
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
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profile_value(name: str, key: str):
    """A figure recorded in a committed ncu summary under profiles/ ('key: value')."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def gbs(nbytes: float, ms: float) -> float:
    return nbytes / (ms / 1e3) / 1e9


# ---------------------------------------------------------------------------
# ranks, barriers and device timing
# ---------------------------------------------------------------------------
class Ctx:
    """One rank of the benchmark: its device and the timing conventions
    (barrier + synchronize on both sides, CUDA events on the launching stream,
    max over ranks)."""

    def __init__(self, args, rank: int, world: int, local_rank: int):
        import torch
        self.a, self.rank, self.world, self.local_rank = args, rank, world, local_rank
        self.dev = torch.device(f"cuda:{local_rank}")
        torch.cuda.set_device(self.dev)
        self.stream = torch.cuda.current_stream(self.dev)

    def barrier(self):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max(self, x: float) -> float:
        """Max over ranks (a collective: every rank calls it in the same order)."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return float(x)
        t = torch.tensor([float(x)], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_ms(self, fn, reps: int) -> float:
        """Device time of reps calls of fn, max over ranks, barrier both sides."""
        import torch
        self.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for i in range(reps):
            fn(i)
        e1.record(self.stream)
        self.barrier()
        return self.max(e0.elapsed_time(e1))


def timed_steps(ctx: Ctx, step, steps: int, warmup: int, before=None, graph: bool = True):
    """Warm-up steps run eagerly; then the step is captured into a CUDA graph
    (two steps per graph on several GPUs, so that each exchange's epoch parity
    still alternates from replay to replay) and exactly `steps` steps are timed
    by replaying it, as a serving loop would run a fixed-shape step; the
    kernels are the same, the per-launch host overhead is gone. Returns (total
    ms max over ranks, clocks, graph)."""
    import torch
    for _ in range(max(3, warmup)):
        step()
    ctx.barrier()
    per = 2 if ctx.world > 1 else 1
    g = None
    run = lambda i: step()  # noqa: E731
    reps = steps
    if graph and steps % per == 0:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(per):
                step()
        g.replay()  # one untimed replay
        ctx.barrier()
        run = lambda i: g.replay()  # noqa: E731
        reps = steps // per
    if before is not None:
        before()
    sampler = ClockSampler(ctx.local_rank)
    sampler.start()
    time.sleep(0.3)
    ms = ctx.time_ms(run, reps)
    return ms, sampler.stop(), g


def check_status(ctx: Ctx, what: str, words: dict) -> dict:
    """Refuse a bench line from a run in which a kernel gave up a bounded wait."""
    vals = {k: int(v.item()) for k, v in words.items() if v is not None}
    bad = {k: v for k, v in vals.items() if v}
    if bad:
        raise SystemExit(f"rank {ctx.rank}: {what}: kernel status words nonzero {bad}; no line")
    return vals


# ---------------------------------------------------------------------------
# CPU baseline: the reference's CPU path (restated in oracle/), one whole
# layer per sample, extrapolated over the layers only
# ---------------------------------------------------------------------------
_cpu_cache: dict = {}


def cpu_threads() -> int:
    import torch
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    return cores


def _cpu_inputs(key, make):
    if key not in _cpu_cache:
        _cpu_cache[key] = make()
    return _cpu_cache[key]


def cpu_cfg3(a, reps: int = 2) -> dict:
    """One layer of the verify attention as ONE torch.sdpa call over all B*T
    rows with the [B*T, P+B*T] tree mask (fp32), the acceptance walk over the
    full logits, and the cat commit of one layer; step = L x (layer +
    commit) + walk."""
    import numpy as np
    import torch

    from oracle import accept as OA
    from oracle import attention as AT
    from oracle import commit as OC
    cores = cpu_threads()
    Hq, Hk, D, V = CFG3["qo_heads"], CFG3["kv_heads"], CFG3["head_dim"], CFG3["vocab"]
    P, T, B = a.prefix, a.block, a.branches

    def make():
        g = torch.Generator().manual_seed(0)
        z = torch.randn(B, T, V, generator=g)
        x = torch.randint(0, V, (B, T), generator=g)
        x[:, 1:] = torch.where(torch.rand(B, T - 1, generator=g) < 0.7, z.argmax(-1)[:, :-1],
                               x[:, 1:])
        return (torch.randn(B, T, Hq, D, generator=g), torch.randn(B, T, Hk, D, generator=g),
                torch.randn(B, T, Hk, D, generator=g), torch.randn(P, Hk, D, generator=g),
                torch.randn(P, Hk, D, generator=g), z.numpy(), x.numpy(),
                np.zeros((1, Hk, P, D), np.float32),
                np.random.default_rng(1).standard_normal((B, Hk, T, D)).astype(np.float32))
    q, kn, vn, kp, vp, zn, xn, cache_k, new = _cpu_inputs(("cfg3", P, B, T), make)
    t_att, t_acc, t_com = [], [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        AT.torch_tree_sdpa(q, kn, vn, kp, vp, causal=True)
        t1 = time.perf_counter()
        acc, _, br = OA.verify_accept(zn, xn)
        t2 = time.perf_counter()
        OC.commit_contiguous([cache_k], [cache_k], [(new, new)], br, acc)
        t3 = time.perf_counter()
        t_att.append(t1 - t0)
        t_acc.append(t2 - t1)
        t_com.append(t3 - t2)
    att, acc_t, com = (statistics.median(v) for v in (t_att, t_acc, t_com))
    step = a.layers * (att + com) + acc_t
    return {"value": B * T / step, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"median of {reps} x [one whole layer: one fp32 torch.sdpa over all {B * T} "
                       f"rows with the [{B * T}, {P}+{B * T}] tree mask ({Hq}/{Hk} heads, D {D}), "
                       f"the cat commit of that layer, the acceptance walk over [{B},{T},{V}] "
                       f"fp32 logits]; step = {a.layers} x (layer + commit) + walk"),
            "seconds_per_step": step}


def cfg4_lengths() -> list[int]:
    import numpy as np
    return np.random.default_rng(CFG4["seed"]).integers(
        CFG4["prefix_lo"], CFG4["prefix_hi"] + 1, CFG4["requests"]).tolist()


def cpu_cfg4(reps: int = 1) -> dict:
    """One layer of all 64 requests' attention (a tree-masked sdpa per
    request), their cat commits and the 64 acceptance walks; step = L x
    (layer + commits) + walks."""
    import numpy as np
    import torch

    from oracle import accept as OA
    from oracle import attention as AT
    from oracle import commit as OC
    cores = cpu_threads()
    c = CFG4
    lens, B, T, Hq, Hk, D, V = (cfg4_lengths(), c["branches"], c["block"], c["qo_heads"],
                                c["kv_heads"], c["head_dim"], c["vocab"])

    def make():
        g = torch.Generator().manual_seed(0)
        reqs = [(torch.randn(B, T, Hq, D, generator=g), torch.randn(B, T, Hk, D, generator=g),
                 torch.randn(B, T, Hk, D, generator=g), torch.randn(P, Hk, D, generator=g),
                 torch.randn(P, Hk, D, generator=g)) for P in lens]
        z = torch.randn(B, T, V, generator=g).numpy()  # one logits block, walked 64 times
        x = np.random.default_rng(0).integers(0, V, (B, T))
        new = np.random.default_rng(1).standard_normal((B, Hk, T, D)).astype(np.float32)
        caches = [np.zeros((1, Hk, P, D), np.float32) for P in lens]
        return reqs, z, x, new, caches
    reqs, z, x, new, caches = _cpu_inputs("cfg4", make)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for (q, kn, vn, kp, vp) in reqs:
            AT.torch_tree_sdpa(q, kn, vn, kp, vp, causal=True)
        t1 = time.perf_counter()
        for ck in caches:
            OC.commit_contiguous([ck], [ck], [(new, new)], 0, 5)
        t2 = time.perf_counter()
        for _r in lens:
            OA.verify_accept(z, x)
        t3 = time.perf_counter()
        ts.append((t1 - t0, t2 - t1, t3 - t2))
    att, com, acc = (statistics.median(v[i] for v in ts) for i in range(3))
    step = c["layers"] * (att + com) + acc
    return {"value": len(lens) * B * T / step, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"median of {reps} x [one whole layer of all {len(lens)} requests: a "
                       f"tree-masked fp32 torch.sdpa per request, their cat commits, and "
                       f"{len(lens)} acceptance walks over [{B},{T},{V}] fp32 logits]; step = "
                       f"{c['layers']} x (layer + commits) + walks"),
            "seconds_per_step": step}


def cpu_cfg5(reps: int = 3) -> dict:
    """One full and one sliding-window layer (the reference truncates the
    prefix to the last `window` keys), the sink rescale, the commits and the
    walk over V 201088; step = L/2 x (full + sliding) + walk."""
    import numpy as np
    import torch

    from oracle import accept as OA
    from oracle import attention as AT
    from oracle import commit as OC
    cores = cpu_threads()
    c = CFG5
    P, B, T, Hq, Hk, D, V, W = (c["prefix"], c["branches"], c["block"], c["qo_heads"],
                                c["kv_heads"], c["head_dim"], c["vocab"], c["window"])

    def make():
        g = torch.Generator().manual_seed(0)
        return (torch.randn(B, T, Hq, D, generator=g), torch.randn(B, T, Hk, D, generator=g),
                torch.randn(B, T, Hk, D, generator=g), torch.randn(P, Hk, D, generator=g),
                torch.randn(P, Hk, D, generator=g), torch.randn(Hq, generator=g),
                torch.randn(B, T, V, generator=g).numpy(),
                np.random.default_rng(0).integers(0, V, (B, T)),
                np.zeros((1, Hk, P, D), np.float32),
                np.random.default_rng(1).standard_normal((B, Hk, T, D)).astype(np.float32))
    q, kn, vn, kp, vp, sinks, z, x, ck, new = _cpu_inputs("cfg5", make)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for kpl, vpl in ((kp, vp), (kp[-W:], vp[-W:])):
            o = AT.torch_tree_sdpa(q, kn, vn, kpl, vpl, causal=True)
            o = o * torch.sigmoid(sinks.view(1, 1, Hq, 1))  # the sink factor's elementwise pass
            OC.commit_contiguous([ck], [ck], [(new, new)], 0, 5)
        t1 = time.perf_counter()
        OA.verify_accept(z, x)
        t2 = time.perf_counter()
        ts.append((t1 - t0, t2 - t1))
    pair, acc = (statistics.median(v[i] for v in ts) for i in range(2))
    step = c["layers"] // 2 * pair + acc
    return {"value": B * T / step, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"median of {reps} x [one full (P {P}) and one sliding ({W} keys) layer: "
                       f"tree-masked fp32 torch.sdpa, sink rescale, cat commit; the walk over "
                       f"[{B},{T},{V}] fp32 logits]; step = {c['layers'] // 2} x (full + "
                       f"sliding) + walk"),
            "seconds_per_step": step}


def cpu_cfg2(reps: int = 2) -> dict:
    """One Qwen3-8B decoder layer of the verify forward on the CPU (fp32,
    random weights): RMSNorm, q/k/v projections, QK-norm, the tree-masked
    sdpa over the 2048-token prefix + 4 x 32 candidates, o_proj, SwiGLU MLP;
    plus lm_head over the 128 rows and the walk; step = L x layer + lm_head +
    walk."""
    import numpy as np
    import torch
    import torch.nn.functional as F

    from oracle import accept as OA
    from oracle import attention as AT
    cores = cpu_threads()
    c = CFG2
    H, I, Hq, Hk, D, V, P = (c["hidden"], c["intermediate"], c["qo_heads"], c["kv_heads"],
                             c["head_dim"], c["vocab"], c["prefix"])
    B, T = c["branches"], c["block"]
    n = B * T

    def make():
        g = torch.Generator().manual_seed(0)
        w = lambda *s: torch.randn(*s, generator=g) * 0.02  # noqa: E731
        return dict(x=torch.randn(n, H, generator=g), wq=w(Hq * D, H), wk=w(Hk * D, H),
                    wv=w(Hk * D, H), wo=w(H, Hq * D), wg=w(I, H), wu=w(I, H), wd=w(H, I),
                    lm=w(V, H), kp=torch.randn(P, Hk, D, generator=g),
                    vp=torch.randn(P, Hk, D, generator=g),
                    ids=np.random.default_rng(0).integers(0, V, (B, T)))
    m = _cpu_inputs("cfg2", make)

    def rms(t):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)

    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        h = rms(m["x"])
        q = rms((h @ m["wq"].T).view(n, Hq, D))
        k = rms((h @ m["wk"].T).view(n, Hk, D))
        v = (h @ m["wv"].T).view(n, Hk, D)
        o = AT.torch_tree_sdpa(q.view(B, T, Hq, D), k.view(B, T, Hk, D), v.view(B, T, Hk, D),
                               m["kp"], m["vp"], causal=True)
        hid = m["x"] + o.reshape(n, Hq * D) @ m["wo"].T
        h2 = rms(hid)
        hid = hid + (F.silu(h2 @ m["wg"].T) * (h2 @ m["wu"].T)) @ m["wd"].T
        t1 = time.perf_counter()
        logits = (rms(hid) @ m["lm"].T).view(B, T, V)
        OA.verify_accept(logits.numpy(), m["ids"])
        t2 = time.perf_counter()
        ts.append((t1 - t0, t2 - t1))
    layer, head = (statistics.median(v[i] for v in ts) for i in range(2))
    step = c["layers"] * layer + head
    return {"value": n / step, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"median of {reps} x [one fp32 Qwen3-8B decoder layer over {n} candidate "
                       f"rows (projections, QK-norm, tree-masked torch.sdpa over {P}+{n} keys, "
                       f"o_proj, SwiGLU MLP) + lm_head and the walk]; step = {c['layers']} x "
                       f"layer + lm_head + walk (RoPE omitted)"),
            "seconds_per_step": step}


def workload_config(a, n) -> dict:
    return {
        "workload": (f"BASELINE config 3 verify step on Qwen3-8B heads: {a.layers} layers x "
                     f"cascade attention ({CFG3['qo_heads']}q/{CFG3['kv_heads']}kv heads, D "
                     f"{CFG3['head_dim']}, prefix {a.prefix} paged (page {CFG3['page_size']}), "
                     f"{a.branches} branches x {a.block} tokens, tree trunk k={a.shared}) + greedy "
                     f"acceptance over [{a.branches},{a.block},{CFG3['vocab']}] bf16 logits + KV "
                     f"commit into {a.layers} layers"),
        "global_batch": a.branches * a.block,
        "seq_len": a.prefix,
        "parallelism": (f"kv-head shard x{n}, per-layer output all-gather "
                        + ("by kernel (b)'s NVLink stores" if a.exchange == "peer" else "by NCCL")
                        + ", vocabulary-sharded acceptance" if n > 1 else "single GPU"),
        "l2": "inputs larger than L2 (paged KV of all layers streamed each step)",
        "kv_pages": ("16-key pages in tensor-core core-matrix order" if a.kv_layout == "umma"
                     else "16-key pages of plain rows [page, head, slot, dim]"),
    }


def run_reference(a, rank: int, world: int):
    """The reference arm: the CPU path of config 3, one bounded sample (one
    whole layer) per step, on rank 0 only."""
    if rank != 0:
        return
    for _ in range(max(0, a.warmup)):
        cpu_cfg3(a, reps=1)
    vals = []
    t0 = time.perf_counter()
    res = None
    for _ in range(a.steps):
        res = cpu_cfg3(a, reps=1)
        vals.append(res["seconds_per_step"])
    wall = time.perf_counter() - t0
    step = statistics.median(vals)
    value = a.branches * a.block / step
    line = {
        "impl": "reference", "metric": "verified tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(a, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": res["cores"],
                         "kind": "port", "sample": res["sample"].replace("median of 1 x ", "")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "wall_s": wall,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# config 3 (the headline)
# ---------------------------------------------------------------------------
class Cfg3:
    """State of the config-3 verify step on one rank: its kv heads' paged
    cache of every layer, the block's q/k/v per layer, the logits (its
    vocabulary slice when sharded), and the kernels' workspaces."""

    def __init__(self, ctx: Ctx):
        import torch

        import d2sd_b200 as d
        a, dev, world, rank = ctx.a, ctx.dev, ctx.world, ctx.rank
        self.ctx = ctx
        L, P, B, T = a.layers, a.prefix, a.branches, a.block
        Hq, Hk, D, V = CFG3["qo_heads"], CFG3["kv_heads"], CFG3["head_dim"], CFG3["vocab"]
        if Hk % world:
            raise SystemExit(f"{Hk} kv heads do not shard over {world} GPUs")
        self.L, self.P, self.B, self.T, self.V, self.D = L, P, B, T, V, D
        self.hk, self.hq = Hk // world, Hq // world
        hk, hq = self.hk, self.hq
        self.N = N = B * T
        self.n_u = a.shared + B * (T - a.shared) if a.shared else N
        self.scale = D ** -0.5
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        self.cache = d.PagedKVCache(L, hk, D, P + T + 16, device=dev, layout=a.kv_layout,
                                    page_order=torch.randperm(-(-(P + T + 16) // 16),
                                                              generator=torch.Generator().manual_seed(7)))
        self.cache.k.normal_(generator=g)
        self.cache.v.normal_(generator=g)
        self.cache.length = P
        q = torch.randn(L, B, T, hq, D, generator=g, device=dev).to(torch.bfloat16)
        if a.shared:
            q[:, :, :a.shared] = q[:, 0:1, :a.shared]
        self.kn = torch.randn(L, B, T, hk, D, generator=g, device=dev).to(torch.bfloat16)
        self.vn = torch.randn(L, B, T, hk, D, generator=g, device=dev).to(torch.bfloat16)
        gz = torch.Generator(device=dev).manual_seed(99)  # the same logits on every rank
        logits = torch.randn(B, T, V, generator=gz, device=dev).to(torch.bfloat16)
        ids = torch.randint(0, V, (B, T), generator=gz, device=dev)
        keep = torch.rand(B, T, generator=gz, device=dev) < 0.7
        ids[:, 1:] = torch.where(keep[:, 1:], logits.float().argmax(-1)[:, :-1], ids[:, 1:])
        ids[:, 0] = ids[0, 0]
        self.ids = ids.view(1, B, T)
        self.plan = d.CascadePlan([d.Request(self.n_u, 0, 0, P)], hq, hk, D, dev)
        self.ptok = d.shared_trunk_map(B, T, a.shared, dev) if a.shared else None
        self.q_pref = [torch.cat([q[l, 0, :a.shared], q[l, :, a.shared:].reshape(-1, hq, D)], 0)
                       if a.shared else q[l].reshape(N, hq, D) for l in range(L)]
        self.q_full = [q[l].reshape(N, hq, D) for l in range(L)]
        self.kns = [self.kn[l] for l in range(L)]
        self.vns = [self.vn[l] for l in range(L)]
        self.out = torch.empty(N, hq, D, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(N, hq, dtype=torch.float32, device=dev)
        self.gathered = (torch.empty(world * N, hq, D, dtype=torch.bfloat16, device=dev)
                         if world > 1 and a.exchange == "nccl" else None)
        self.px = (d.PeerExchange(N, Hq, Hk, D, torch.bfloat16, dev)
                   if world > 1 and a.exchange == "peer" else None)
        if world > 1:
            self.ver = d.ShardedVerifier(1, B, T, V, dev)
            c0, c1 = self.ver.columns
            self.logits = logits[..., c0:c1].contiguous().view(1, B, T, c1 - c0)
        else:
            self.ver = d.BatchVerifier(1, B, T, V, dev)
            self.logits = logits.view(1, B, T, V)
        self.full_logits_bytes = B * T * V * 2
        self.new_k = self.kn.transpose(2, 3)  # [L, B, hk, T, D] views of the token-major K/V
        self.new_v = self.vn.transpose(2, 3)
        self.bstatus = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ev = None

    def mark(self, name):
        import torch
        if self.ev is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(self.ctx.stream)
            self.ev[name].append(e)

    def attention(self, l, qp, qf, kn, vn):
        self.plan.run_prefix(qp, self.cache.k[l], self.cache.v[l], self.cache.kv_layout,
                             self.scale, page_table=self.cache.page_table)
        self.mark("a1")
        self.suffix(qf, kn, vn)

    def suffix(self, qf, kn, vn):
        import torch.distributed as dist

        from d2sd_b200 import ops
        N, hq, hk, D = self.N, self.hq, self.hk, self.D
        ops.suffix_merge(qf, kn.reshape(N, hk, D), vn.reshape(N, hk, D), self.out, self.lse,
                         num_blocks=self.B, block_len=self.T, num_qo_heads=hq, num_kv_heads=hk,
                         sm_scale=self.scale, partial=self.plan.partial, plan_dev=self.plan.plan,
                         prefix_token=self.ptok, exchange=self.px, status=self.bstatus)
        if self.gathered is not None:
            dist.all_gather_into_tensor(self.gathered, self.out)

    def step(self, qp=None, qf=None, kns=None, vns=None, logits=None, ids=None,
             wait_layer=None, wait_logits=None):
        qp, qf = qp or self.q_pref, qf or self.q_full
        kns, vns = kns or self.kns, vns or self.vns
        for l in range(self.L):
            if wait_layer is not None:
                wait_layer(l)
            self.mark("a0")
            self.attention(l, qp[l], qf[l], kns[l], vns[l])
            self.mark("b1")
        self.mark("c0")
        if wait_logits is not None:
            wait_logits()
        self.ver.launch(self.logits if logits is None else logits,
                        self.ids if ids is None else ids)
        self.mark("c1")
        self.cache.commit(self.new_k, self.new_v, self.ver.result[0], cache_len=self.P)
        self.mark("d1")

    def run_a(self, l):
        self.plan.run_prefix(self.q_pref[l], self.cache.k[l], self.cache.v[l],
                             self.cache.kv_layout, self.scale, page_table=self.cache.page_table)

    def run_ab(self, l):
        self.attention(l, self.q_pref[l], self.q_full[l], self.kns[l], self.vns[l])

    def run_b(self, l):
        self.suffix(self.q_full[l], self.kns[l], self.vns[l])

    def run_c(self):
        self.ver.launch(self.logits, self.ids)

    def run_d(self):
        self.cache.commit(self.new_k, self.new_v, self.ver.result[0], cache_len=self.P)

    def statuses(self):
        words = {"a": self.plan.status, "b": self.bstatus}
        if self.px is not None:
            words["exchange"] = self.px.status
        if self.ctx.world > 1:
            words["accept_exchange"] = self.ver.status
        return words

    def close(self):
        if self.px is not None:
            self.px.close()
        if self.ctx.world > 1:
            self.ver.close()


def bench_cfg3(ctx: Ctx) -> dict:
    """The headline line: device-resident timing, per-kernel and back-to-back
    times, the roofline of kernel (a), then the end-to-end run."""
    import torch
    a = ctx.a
    c = Cfg3(ctx)
    L, N = c.L, c.N
    before = c.px.reset_stats if c.px is not None else None
    ms_total, clocks, graph = timed_steps(ctx, c.step, a.steps, a.warmup, before,
                                          graph=a.exchange == "peer" or ctx.world == 1)
    ms_step = ms_total / a.steps
    xwait = c.px.wait_stats() if c.px is not None else None
    del graph
    # kernel (a)'s launches with their launch gaps: events around each launch
    # of one eager step after the timed region (an event between two kernels
    # also stops the programmatic launch overlap)
    c.ev = {k: [] for k in ("a0", "a1", "b1", "c0", "c1", "d1")}
    c.step()
    ctx.barrier()
    ev, c.ev = c.ev, None
    a_marked = ctx.max(statistics.mean(s.elapsed_time(e) for s, e in zip(ev["a0"], ev["a1"])))
    acc_len = int(c.ver.result[0, 0].item())
    k = kernel_ms(ctx, c)
    a_b2b, ab_b2b, c_avg, d_avg, b_avg = k["a"], k["ab"], k["c"], k["d"], k["b"]
    statuses = check_status(ctx, "config 3", c.statuses())

    hbm, tf_burst, tf_sust, peak_src = measured_peaks()
    P, D, hq, hk = c.P, c.D, c.hq, c.hk
    flops_a = 4.0 * c.n_u * hq * P * D
    achieved = flops_a / (a_b2b / 1e3) / 1e12
    achieved_marked = flops_a / (a_marked / 1e3) / 1e12
    prof = "prefix_attention_cfg3.txt"
    full_shape = ctx.world == 1 and P == 32768 and not a.shared and a.kv_layout == "umma"
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
        "frac": achieved / tf_burst,
        "traffic": profile_value(prof, "traffic_bytes_per_launch") if full_shape else None,
        "achieved_per_marked_launch": achieved_marked,
        "frac_per_marked_launch": achieved_marked / tf_burst,
        "ncu_tensor_pipe_active": profile_value(prof, "tensor_pipe_active") if full_shape else None,
        "frac_of_sustained": achieved / tf_sust,
        "timing": ("achieved: kernel (a) back to back over all layers from a CUDA graph (as in "
                   "the timed step), CUDA events around the replay; per_marked_launch: events "
                   "around each launch of an eager step (includes each launch's latency)"),
        "peak_source": (f"bf16_tflops (burst) of {peak_src}: the timed region lasts "
                        f"{ms_total / 1e3:.2f} s at full clock"),
        "kernel": "prefix_attention_kernel (a)",
        "algorithmic": f"4*N_u*Hq*P*D = {flops_a:.4g} FLOP per launch",
    }
    slot_b = c.plan.partial.numel() * c.plan.partial.element_size() if c.plan.num_slots else 0
    bytes_b = N * hq * D * 2 + 2 * N * hk * D * 2 + N * hq * D * 2 + N * hq * 4 + slot_b
    bytes_c = c.logits.numel() * 2 + N * 8
    bytes_d = 2 * acc_len * L * 2 * hk * D * 2
    kernels = {
        "a_prefix_attention_us": a_b2b * 1e3, "a_per_marked_launch_us": a_marked * 1e3,
        "a_hbm_floor_us": 2 * P * hk * D * 2 / (hbm * 1e9) * 1e6,
        "b_suffix_merge_us": b_avg * 1e3, "b_suffix_merge_gbs": gbs(bytes_b, b_avg),
        "c_accept_us": c_avg * 1e3, "c_accept_gbs": gbs(bytes_c, c_avg),
        "d_commit_us": d_avg * 1e3, "d_commit_gbs": gbs(bytes_d, d_avg),
        "hbm_peak_gbs": hbm,
        "hbm_frac": {"b": gbs(bytes_b, b_avg) / hbm, "c": gbs(bytes_c, c_avg) / hbm,
                     "d": gbs(bytes_d, d_avg) / hbm},
        "ab_back_to_back_us": ab_b2b * 1e3, "b_marginal_us": k["b_marginal"] * 1e3,
        "timing": "each kernel back to back from a CUDA graph of repeated launches; b = (a+b) - a",
        "acceptance_length": acc_len,
    }
    out = {"value": N * a.steps / (ms_total / 1e3), "ms_per_step": ms_step,
           "step_timing": ("the step captured into a CUDA graph (two steps per graph on several "
                           "GPUs) and replayed; warm-up, per-kernel events and e2e run eagerly"),
           "us_per_layer": (ms_step - c_avg - d_avg) / L * 1e3, "status": statuses,
           "roofline": roofline, "kernels": kernels, "clocks": clocks,
           "gpu_launches": a.steps * (2 * L + 2)}
    if xwait is not None:
        # time the signalling CTA of kernel (b) waited for the other ranks, per
        # layer, in the timed region (the worst rank's mean and maximum)
        out["exchange_wait"] = {"mean_us_per_layer": ctx.max(xwait["mean_wait_us"]),
                                "max_us": ctx.max(xwait["max_wait_us"]), "waits": xwait["waits"]}
    if not a.no_e2e:
        out["e2e"] = e2e_cfg3(ctx, c)
    if a.flashinfer and ctx.world == 1:
        out["flashinfer"] = flashinfer_cfg3(ctx, c, ab_b2b)
    ctx.barrier()  # no kernel of any rank is still using the peer buffers
    c.close()
    ctx.barrier()  # every rank has unmapped its peers' buffers before they are freed
    del c
    torch.cuda.empty_cache()
    return out


def bench_cfg3_trunk(ctx: Ctx, shared: int) -> dict:
    """Config 3 with a tree whose branches share their first `shared` tokens
    (N_u = k + B*(T-k) unique query rows in kernel (a)): the step timed as the
    headline's, and kernel (a)'s roofline on the unique rows."""
    import copy

    import torch
    a2 = copy.copy(ctx.a)
    a2.shared = shared
    ctx2 = copy.copy(ctx)
    ctx2.a = a2
    c = Cfg3(ctx2)
    ms_total, clocks, graph = timed_steps(ctx2, c.step, a2.steps, a2.warmup)
    del graph
    k = kernel_ms(ctx2, c)
    statuses = check_status(ctx2, f"config 3, trunk {shared}", c.statuses())
    _, tf_burst, _, peak_src = measured_peaks()
    flops = 4.0 * c.n_u * c.hq * c.P * c.D
    achieved = flops / (k["a"] / 1e3) / 1e12
    out = {"metric": "verified tokens/s", "unit": "tokens/s",
           "value": c.N * a2.steps / (ms_total / 1e3), "ms_per_step": ms_total / a2.steps,
           "shared_trunk": shared, "unique_query_tokens": c.n_u, "status": statuses,
           "clocks": clocks,
           "roofline": {"bound": "tensor", "kernel": "prefix_attention_kernel (a)",
                        "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
                        "frac": achieved / tf_burst, "peak_source": f"bf16_tflops of {peak_src}",
                        "algorithmic": f"4*N_u*Hq*P*D = {flops:.4g} FLOP per launch"},
           "kernels": {"a_prefix_attention_us": k["a"] * 1e3, "b_marginal_us": k["b_marginal"] * 1e3,
                       "c_accept_us": k["c"] * 1e3, "d_commit_us": k["d"] * 1e3},
           "gpu_launches": a2.steps * (2 * c.L + 2)}
    c.close()
    del c
    torch.cuda.empty_cache()
    return out


def e2e_cfg3(ctx: Ctx, c: Cfg3) -> dict:
    """The same step through the public API from pinned host buffers: each
    step copies every layer's q/k/v (this rank's heads) and the logits (this
    rank's vocabulary slice) host->device on a copy stream, layer l's attention
    waiting only for layer l's inputs, and reads the result back."""
    import torch
    a, dev, stream = ctx.a, ctx.dev, ctx.stream
    L, N, hq, D = c.L, c.N, c.hq, c.D
    pin = lambda t: t.cpu().pin_memory()  # noqa: E731
    h_qp, h_kn, h_vn = [pin(t) for t in c.q_pref], [pin(t) for t in c.kns], [pin(t) for t in c.vns]
    h_qf = [pin(t) for t in c.q_full] if a.shared else None
    h_logits, h_ids = pin(c.logits), pin(c.ids)
    d_qp = [torch.empty_like(t) for t in c.q_pref]
    d_qf = [torch.empty_like(t) for t in c.q_full] if a.shared else None
    d_kn, d_vn = [torch.empty_like(t) for t in c.kns], [torch.empty_like(t) for t in c.vns]
    d_logits, d_ids = torch.empty_like(c.logits), torch.empty_like(c.ids)
    h_res = torch.empty(2, dtype=torch.int32).pin_memory()
    h_acc = torch.empty(c.T, dtype=torch.int64).pin_memory()
    nb = lambda ts: sum(t.numel() * t.element_size() for t in ts)  # noqa: E731
    h2d = nb(h_qp + h_kn + h_vn + [h_logits, h_ids]) + (nb(h_qf) if a.shared else 0)
    d2h = h_res.numel() * 4 + h_acc.numel() * 8
    copy_stream = torch.cuda.Stream(dev)
    ev_layer = [torch.cuda.Event() for _ in range(L)]
    ev_logits = torch.cuda.Event()
    qf = d_qf if a.shared else [t.view(N, hq, D) for t in d_qp]

    def e2e_step(_i):
        copy_stream.wait_stream(stream)  # after the timer start and the previous step
        with torch.cuda.stream(copy_stream):
            for l in range(L):
                d_qp[l].copy_(h_qp[l], non_blocking=True)
                if a.shared:
                    d_qf[l].copy_(h_qf[l], non_blocking=True)
                d_kn[l].copy_(h_kn[l], non_blocking=True)
                d_vn[l].copy_(h_vn[l], non_blocking=True)
                ev_layer[l].record(copy_stream)
            d_logits.copy_(h_logits, non_blocking=True)
            d_ids.copy_(h_ids, non_blocking=True)
            ev_logits.record(copy_stream)
        c.step(d_qp, qf, d_kn, d_vn, d_logits, d_ids,
               wait_layer=lambda l: stream.wait_event(ev_layer[l]),
               wait_logits=lambda: stream.wait_event(ev_logits))
        h_res.copy_(c.ver.result[0], non_blocking=True)
        h_acc.copy_(c.ver.accepted[0], non_blocking=True)
        stream.synchronize()

    for i in range(max(3, a.warmup)):
        e2e_step(i)
    e_ms = ctx.time_ms(e2e_step, a.steps)
    check_status(ctx, "config 3 end to end", c.statuses())
    return {"value": N * a.steps / (e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": e_ms / a.steps}


def flashinfer_cfg3(ctx: Ctx, c: Cfg3, ab_ms: float) -> dict:
    """The reference's own GPU path of one config-3 layer on the same inputs,
    as generation/verification.py:139-165 and model/cascade_graph.py:37-112
    run it: the DynamicCache [Hk, P, D] prefix transposed to NHD, FlashInfer's
    single_prefill_with_kv_cache over it (level 1), then the runner's copies
    in, B x (causal single_prefill + merge_state_in_place) and copies out.
    Everything is captured in one CUDA graph (the reference runs level 1
    eagerly: this favours it). Also a second parity reference: FlashInfer's
    merged output against kernels (a)+(b) on the same layer."""
    import torch
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer import failed: {type(e).__name__}: {e}"}
    B, T, N, hq, hk, D, P = c.B, c.T, c.N, c.hq, c.hk, c.D, c.P
    if c.ctx.a.shared:
        return {"unavailable": "the reference path has no shared-trunk form"}
    k_tok, v_tok = c.cache.gather(0, P)
    k_hnd, v_hnd = k_tok.transpose(0, 1).contiguous(), v_tok.transpose(0, 1).contiguous()
    del k_tok, v_tok
    q_all = c.q_full[0]                      # [B*T, Hq, D]
    q_fi = q_all.view(B, T, hq, D)
    kn, vn = c.kn[0], c.vn[0]                # [B, T, Hk, D]
    k_new = kn.transpose(1, 2)               # the projections' [B, Hk, T, D] view
    v_new = vn.transpose(1, 2)
    bufs = {n: torch.empty_like(t) for n, t in (("q", q_fi), ("k", kn), ("v", vn))}
    bufs["out"] = torch.empty(B, T, hq, D, dtype=torch.bfloat16, device=ctx.dev)
    bufs["lse"] = torch.empty(B, T, hq, dtype=torch.float32, device=ctx.dev)
    res = {}

    def level1():
        kf = k_hnd.transpose(0, 1).contiguous()
        vf = v_hnd.transpose(0, 1).contiguous()
        o, s = flashinfer.single_prefill_with_kv_cache(q_all, kf, vf, causal=False,
                                                       return_lse=True, sm_scale=c.scale)
        res["o"], res["s"] = o.view(B, T, hq, D), s.view(B, T, hq)

    def local_merge():
        for i in range(B):
            ol, sl = flashinfer.single_prefill_with_kv_cache(
                bufs["q"][i], bufs["k"][i], bufs["v"][i], causal=True, return_lse=True,
                sm_scale=c.scale)
            flashinfer.merge_state_in_place(bufs["out"][i], bufs["lse"][i], ol, sl)

    def layer():
        level1()
        k_fi, v_fi = k_new.transpose(1, 2).contiguous(), v_new.transpose(1, 2).contiguous()
        bufs["q"].copy_(q_fi)
        bufs["k"].copy_(k_fi)
        bufs["v"].copy_(v_fi)
        bufs["out"].copy_(res["o"])
        bufs["lse"].copy_(res["s"])
        local_merge()
        res["o"].copy_(bufs["out"])
        res["s"].copy_(bufs["lse"])

    def prefill_only():
        flashinfer.single_prefill_with_kv_cache(q_all, k_tok_nhd, v_tok_nhd, causal=False,
                                                return_lse=True, sm_scale=c.scale)

    try:
        t0 = time.perf_counter()
        for _ in range(3):  # JIT compile + warm-up, eagerly
            layer()
        torch.cuda.synchronize()
        compile_s = time.perf_counter() - t0
        k_tok_nhd, v_tok_nhd = k_hnd.transpose(0, 1).contiguous(), v_hnd.transpose(0, 1).contiguous()
        prefill_only()
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer failed: {type(e).__name__}: {str(e)[:300]}"}
    layer_ms = graph_ms(ctx, lambda i: layer(), 8)
    prefill_ms = graph_ms(ctx, lambda i: prefill_only(), 8)
    transpose_ms = graph_ms(ctx, lambda i: (k_hnd.transpose(0, 1).contiguous(),
                                           v_hnd.transpose(0, 1).contiguous()), 8)
    # parity: FlashInfer's merged layer-0 output against kernels (a)+(b)
    layer()
    c.run_ab(0)
    torch.cuda.synchronize()
    ours_o, ours_s = c.out.float().view(B, T, hq, D), c.lse.view(B, T, hq)
    fo, fs = res["o"].float(), res["s"]
    err = (ours_o - fo).abs()
    within = (err <= 2e-2 + 1e-2 * fo.abs()).float().mean().item()
    flops = 4.0 * N * hq * P * D
    hbm, tf_burst, _, _ = measured_peaks()
    out = {
        "what": ("the reference's GPU path of one layer (verification.py:139-165 with the "
                 "CascadeGraphRunner): prefix transpose copy, FlashInfer single_prefill (level 1), "
                 "runner copies, 8 x (causal single_prefill + merge_state_in_place); one CUDA graph"),
        "flashinfer_version": getattr(flashinfer, "__version__", "?"),
        "jit_and_warmup_s": compile_s,
        "layer_us": layer_ms * 1e3,
        "single_prefill_us": prefill_ms * 1e3,
        "single_prefill_tflops": flops / (prefill_ms / 1e3) / 1e12,
        "single_prefill_frac_of_burst_bf16": flops / (prefill_ms / 1e3) / 1e12 / tf_burst,
        "transpose_copy_us": transpose_ms * 1e3,
        "d2sd_ab_us": ab_ms * 1e3,
        "layer_speedup": layer_ms / ab_ms,
        "parity_vs_d2sd": {"max_abs_out": err.max().item(),
                           "max_abs_lse": (ours_s - fs).abs().max().item(),
                           "frac_within_2e-2_abs_1e-2_rel": within},
    }
    del k_hnd, v_hnd, k_tok_nhd, v_tok_nhd, bufs, res
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# config 4: batched serving, request-parallel
# ---------------------------------------------------------------------------
class Cfg4:
    """This rank's share of the 64 requests (LPT on prefix x tokens): their
    caches of every layer in one page pool, one multi-request plan, the
    batched acceptance over their logits and the batched commit."""

    def __init__(self, ctx: Ctx):
        import torch

        import d2sd_b200 as d
        from d2sd_b200.sharding import lpt_partition, request_costs
        c, dev = CFG4, ctx.dev
        self.ctx = ctx
        self.L, self.B, self.T, self.Hq, self.Hk, self.D, self.V = (
            ctx.a.sub_layers or c["layers"], c["branches"], c["block"], c["qo_heads"],
            c["kv_heads"], c["head_dim"], c["vocab"])
        L, B, T, Hq, Hk, D, V = self.L, self.B, self.T, self.Hq, self.Hk, self.D, self.V
        lens = cfg4_lengths()
        self.total_requests = len(lens)
        self.mine = lpt_partition(request_costs(lens, [B * T] * len(lens)), ctx.world)[ctx.rank]
        self.lens = [lens[i] for i in self.mine]
        R = self.R = len(self.lens)
        self.N = N = R * B * T
        self.scale = D ** -0.5
        g = torch.Generator(device=dev).manual_seed(4000 + ctx.rank)
        self.pool = d.PagedKVPool(L, Hk, D, [p + T + 16 for p in self.lens], device=dev,
                                  shuffle_seed=7)
        self.pool.k.normal_(generator=g)
        self.pool.v.normal_(generator=g)
        self.pool.set_lengths(self.lens)
        self.q = torch.randn(L, N, Hq, D, generator=g, device=dev).to(torch.bfloat16)
        self.kn = torch.randn(L, N, Hk, D, generator=g, device=dev).to(torch.bfloat16)
        self.vn = torch.randn(L, N, Hk, D, generator=g, device=dev).to(torch.bfloat16)
        self.new_k = self.kn.view(L, R * B, T, Hk, D).transpose(2, 3)
        self.new_v = self.vn.view(L, R * B, T, Hk, D).transpose(2, 3)
        reqs = [d.Request(B * T, i * B * T, 0, p, self.pool.page_offsets_host[i])
                for i, p in enumerate(self.lens)]
        self.plan = d.CascadePlan(reqs, Hq, Hk, D, dev)
        self.logits = torch.randn(R, B, T, V, generator=g, device=dev).to(torch.bfloat16)
        ids = torch.randint(0, V, (R, B, T), generator=g, device=dev)
        keep = torch.rand(R, B, T, generator=g, device=dev) < 0.7
        ids[:, :, 1:] = torch.where(keep[:, :, 1:], self.logits.float().argmax(-1)[:, :, :-1],
                                    ids[:, :, 1:])
        ids[:, :, 0] = ids[:, 0:1, 0]
        self.ids = ids
        self.ver = d.BatchVerifier(R, B, T, V, dev)
        self.out = torch.empty(N, Hq, D, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(N, Hq, dtype=torch.float32, device=dev)
        self.bstatus = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ev = None

    def mark(self, name):
        import torch
        if self.ev is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(self.ctx.stream)
            self.ev[name].append(e)

    def step(self, q=None, kn=None, vn=None, logits=None, ids=None, wait_layer=None,
             wait_logits=None):
        q = self.q if q is None else q
        kn = self.kn if kn is None else kn
        vn = self.vn if vn is None else vn
        for l in range(self.L):
            if wait_layer is not None:
                wait_layer(l)
            self.mark("a0")
            self.run_a(l, q)
            self.mark("a1")
            self.run_b(l, q, kn, vn)
            self.mark("b1")
        self.mark("c0")
        if wait_logits is not None:
            wait_logits()
        self.ver.launch(self.logits if logits is None else logits,
                        self.ids if ids is None else ids)
        self.mark("c1")
        self.run_d()
        self.mark("d1")

    def run_a(self, l, q=None):
        q = self.q if q is None else q
        self.plan.run_prefix(q[l], self.pool.k[l], self.pool.v[l], self.pool.kv_layout,
                             self.scale, page_table=self.pool.page_table)

    def run_b(self, l, q=None, kn=None, vn=None):
        from d2sd_b200 import ops
        q = self.q if q is None else q
        kn = self.kn if kn is None else kn
        vn = self.vn if vn is None else vn
        ops.suffix_merge(q[l], kn[l], vn[l], self.out, self.lse, num_blocks=self.R * self.B,
                         block_len=self.T, num_qo_heads=self.Hq, num_kv_heads=self.Hk,
                         sm_scale=self.scale, partial=self.plan.partial, plan_dev=self.plan.plan,
                         status=self.bstatus)

    def run_ab(self, l):
        self.run_a(l)
        self.run_b(l)

    def run_c(self):
        self.ver.launch(self.logits, self.ids)

    def run_d(self):
        self.pool.commit_batch(self.new_k, self.new_v, self.ver.result, num_branches=self.B)

    def statuses(self):
        return {"a": self.plan.status, "b": self.bstatus}


def graph_ms(ctx: Ctx, fn, n: int) -> float:
    """Device time per call of fn, from a CUDA graph of n consecutive calls
    (n even: exchanges alternate their epoch parity) replayed once untimed
    and once between two events: the kernels run back to back as in the
    timed step, without host launch gaps; max over ranks."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fn(i)
    g.replay()
    ms = ctx.time_ms(lambda i: g.replay(), 1) / n
    del g
    return ms


def kernel_ms(ctx: Ctx, c) -> dict:
    """Per-kernel device times of a config's step: kernel (a) alone over all
    layers, kernel (b) alone over all layers (re-merging the last partial
    states), (a)+(b) over all layers (b's marginal cost beside (a) = the
    difference), acceptance (c) and commit (d) -- each from a CUDA graph of
    repeated launches."""
    L = c.L
    a = graph_ms(ctx, lambda i: c.run_a(i % L), 2 * L)
    ab = graph_ms(ctx, lambda i: c.run_ab(i % L), 2 * L)
    return {"a": a, "b": graph_ms(ctx, lambda i: c.run_b(i % L), 2 * L), "ab": ab,
            "b_marginal": max(ab - a, 0.0),
            "c": graph_ms(ctx, lambda i: c.run_c(), 10),
            "d": graph_ms(ctx, lambda i: c.run_d(), 10)}


def bench_cfg4(ctx: Ctx) -> dict:
    import torch
    a = ctx.a
    c = Cfg4(ctx)
    L, N, B, T, Hq, Hk, D = c.L, c.N, c.B, c.T, c.Hq, c.Hk, c.D
    ms_total, clocks, graph = timed_steps(ctx, c.step, a.steps, a.warmup)
    del graph
    k = kernel_ms(ctx, c)
    a_b2b = k["a"]
    statuses = check_status(ctx, "config 4", c.statuses())
    hbm, tf_burst, _, peak_src = measured_peaks()
    keys = sum(c.lens)
    flops_a = 4.0 * B * T * Hq * D * keys
    bytes_a = 2.0 * keys * Hk * D * 2 + N * Hq * D * 2 + c.plan.num_slots * (128 * D * 2 + 512)
    ach_t = ctx.max(flops_a / (a_b2b / 1e3) / 1e12)
    ach_b = ctx.max(bytes_a / (a_b2b / 1e3) / 1e9)
    bytes_c = c.logits.numel() * 2 + N * 8
    acc = c.ver.result[:, 0].float().mean().item()
    bytes_d = 2 * acc * c.R * L * 2 * Hk * D * 2
    out = {
        "metric": "verified tokens/s", "unit": "tokens/s",
        "value": c.total_requests * B * T * a.steps / (ms_total / 1e3),
        "ms_per_step": ms_total / a.steps, "n_gpus": ctx.world, "scaling": "strong",
        "parallelism": (f"request-parallel x{ctx.world} (LPT on prefix x tokens), no collective"
                        if ctx.world > 1 else "single GPU"),
        "workload": (f"BASELINE config 4: {c.total_requests} requests, prefix ~ U[512, 8192] "
                     f"(seed {CFG4['seed']}, {sum(cfg4_lengths())} keys in all), {B} branches x "
                     f"{T} tokens, {Hq}/{Hk} heads, D {D}, {L} layers of cascade attention over "
                     f"one 16-key UMMA page pool, batched acceptance over [{c.total_requests},"
                     f"{B},{T},{c.V}] bf16 logits, batched commit"),
        "status": statuses, "clocks": clocks,
        "roofline": {
            "bound": "tensor and hbm (arithmetic intensity B*T*G = 256, at the ridge)",
            "kernel": "prefix_attention_kernel (a), multi-request plan",
            "achieved_tflops": ach_t, "peak_tflops": tf_burst, "frac_tensor": ach_t / tf_burst,
            "achieved_gbs": ach_b, "peak_gbs": hbm, "frac_hbm": ach_b / hbm,
            "timing": "kernel (a) back to back over all layers from a CUDA graph, worst rank",
            "algorithmic": (f"4*B*T*Hq*D*sum(P) = {flops_a:.4g} FLOP and "
                            f"{bytes_a:.4g} B (K+V once, Q, partial slots) per launch on rank "
                            f"{ctx.rank}"),
            "peak_source": peak_src,
        },
        "kernels": {"a_prefix_attention_us": k["a"] * 1e3,
                    "b_suffix_merge_us": k["b"] * 1e3, "b_marginal_us": k["b_marginal"] * 1e3,
                    "c_accept_batch_us": k["c"] * 1e3,
                    "c_accept_gbs": gbs(bytes_c, k["c"]), "d_commit_batch_us": k["d"] * 1e3,
                    "d_commit_gbs": gbs(bytes_d, k["d"]),
                    "requests_on_rank0": c.R, "mean_acceptance_length": acc},
        "gpu_launches": a.steps * (2 * L + 2),
    }
    if not a.no_e2e:
        out["e2e"] = e2e_static(ctx, c, [c.q, c.kn, c.vn], [c.logits, c.ids],
                                lambda: (c.ver.result, c.ver.accepted),
                                c.total_requests * B * T, "config 4")
    del c
    torch.cuda.empty_cache()
    return out


def e2e_static(ctx: Ctx, c, per_layer: list, last: list, results, tokens: int, what: str) -> dict:
    """End to end through the same API from pinned host copies of the step's
    inputs, copied every step into the step's own device buffers: per_layer
    tensors [L, ...] layer by layer on a copy stream (layer l's attention waits
    for layer l's inputs only), then `last` (logits, ids); `results()` is read
    back to the host."""
    import torch
    a, dev, stream = ctx.a, ctx.dev, ctx.stream
    L = per_layer[0].shape[0]
    hosts = [t.cpu().pin_memory() for t in per_layer]
    hlast = [t.cpu().pin_memory() for t in last]
    res = results()
    hres = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in res]
    h2d = sum(t.numel() * t.element_size() for t in hosts + hlast)
    d2h = sum(t.numel() * t.element_size() for t in hres)
    copy_stream = torch.cuda.Stream(dev)
    ev_layer = [torch.cuda.Event() for _ in range(L)]
    ev_last = torch.cuda.Event()

    def e2e_step(_i):
        copy_stream.wait_stream(stream)
        with torch.cuda.stream(copy_stream):
            for l in range(L):
                for d_t, h_t in zip(per_layer, hosts):
                    d_t[l].copy_(h_t[l], non_blocking=True)
                ev_layer[l].record(copy_stream)
            for d_t, h_t in zip(last, hlast):
                d_t.copy_(h_t, non_blocking=True)
            ev_last.record(copy_stream)
        c.step(wait_layer=lambda l: stream.wait_event(ev_layer[l]),
               wait_logits=lambda: stream.wait_event(ev_last))
        for h_t, d_t in zip(hres, results()):
            h_t.copy_(d_t, non_blocking=True)
        stream.synchronize()

    for i in range(max(3, a.warmup)):
        e2e_step(i)
    e_ms = ctx.time_ms(e2e_step, a.steps)
    check_status(ctx, what + " end to end", c.statuses())
    return {"value": tokens * a.steps / (e_ms / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e_ms / a.steps}


# ---------------------------------------------------------------------------
# config 5: GPT-OSS-20B attention shapes, KV-head sharded
# ---------------------------------------------------------------------------
class Cfg5:
    """GPT-OSS-20B verify attention on this rank's kv heads: 24 layers, even
    ones with a 128-token sliding window (the reference's truncation of the
    prefix, generation/verification.py:130-135), odd ones full; learned sinks
    (reference formula); acceptance over V 201088 (vocabulary-sharded on
    several GPUs); commit into every layer."""

    def __init__(self, ctx: Ctx):
        import torch

        import d2sd_b200 as d
        c, dev, world, rank = CFG5, ctx.dev, ctx.world, ctx.rank
        self.ctx = ctx
        self.L, self.P, self.B, self.T = (ctx.a.sub_layers or c["layers"], c["prefix"],
                                          c["branches"], c["block"])
        L, P, B, T, D, V, W = self.L, self.P, self.B, self.T, c["head_dim"], c["vocab"], c["window"]
        self.D, self.V, self.W = D, V, W
        if c["kv_heads"] % world:
            raise SystemExit(f"{c['kv_heads']} kv heads do not shard over {world} GPUs")
        self.hk, self.hq = c["kv_heads"] // world, c["qo_heads"] // world
        hk, hq = self.hk, self.hq
        self.N = N = B * T
        self.scale = D ** -0.5
        g = torch.Generator(device=dev).manual_seed(5000 + rank)
        self.cache = d.PagedKVCache(L, hk, D, P + T + 16, device=dev,
                                    page_order=torch.randperm(-(-(P + T + 16) // 16),
                                                              generator=torch.Generator().manual_seed(5)))
        self.cache.k.normal_(generator=g)
        self.cache.v.normal_(generator=g)
        self.q = torch.randn(L, N, hq, D, generator=g, device=dev).to(torch.bfloat16)
        self.kn = torch.randn(L, N, hk, D, generator=g, device=dev).to(torch.bfloat16)
        self.vn = torch.randn(L, N, hk, D, generator=g, device=dev).to(torch.bfloat16)
        self.sinks = torch.randn(L, hq, generator=g, device=dev)
        self.new_k = self.kn.view(L, B, T, hk, D).transpose(2, 3)
        self.new_v = self.vn.view(L, B, T, hk, D).transpose(2, 3)
        self.sliding = [l % 2 == 0 for l in range(L)]
        self.plans = {s: d.CascadePlan([d.Request(N, 0, P - W if s else 0, P)], hq, hk, D, dev)
                      for s in (True, False)}
        gz = torch.Generator(device=dev).manual_seed(55)  # the same logits on every rank
        logits = torch.randn(B, T, V, generator=gz, device=dev).to(torch.bfloat16)
        ids = torch.randint(0, V, (B, T), generator=gz, device=dev)
        keep = torch.rand(B, T, generator=gz, device=dev) < 0.7
        ids[:, 1:] = torch.where(keep[:, 1:], logits.float().argmax(-1)[:, :-1], ids[:, 1:])
        ids[:, 0] = ids[0, 0]
        self.ids = ids.view(1, B, T)
        if world > 1:
            self.ver = d.ShardedVerifier(1, B, T, V, dev)
            c0, c1 = self.ver.columns
            self.logits = logits[..., c0:c1].contiguous().view(1, B, T, c1 - c0)
        else:
            self.ver = d.BatchVerifier(1, B, T, V, dev)
            self.logits = logits.view(1, B, T, V)
        self.px = (d.PeerExchange(N, c["qo_heads"], c["kv_heads"], D, torch.bfloat16, dev)
                   if world > 1 else None)
        self.out = torch.empty(N, hq, D, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(N, hq, dtype=torch.float32, device=dev)
        self.bstatus = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ev = None

    mark = Cfg4.mark

    def attention(self, l, q, kn, vn):
        self.run_a(l, q)
        self.mark("a1")
        self.run_b(l, q, kn, vn)

    def run_a(self, l, q=None):
        plan = self.plans[self.sliding[l]]
        plan.run_prefix(self.q[l] if q is None else q, self.cache.k[l], self.cache.v[l],
                        self.cache.kv_layout, self.scale, page_table=self.cache.page_table)

    def run_b(self, l, q=None, kn=None, vn=None):
        from d2sd_b200 import _lib, ops
        plan = self.plans[self.sliding[l]]
        ops.suffix_merge(self.q[l] if q is None else q, self.kn[l] if kn is None else kn,
                         self.vn[l] if vn is None else vn, self.out, self.lse,
                         num_blocks=self.B, block_len=self.T, num_qo_heads=self.hq,
                         num_kv_heads=self.hk, sm_scale=self.scale, partial=plan.partial,
                         plan_dev=plan.plan, sinks=self.sinks[l], sink_mode=_lib.SINK_REFERENCE,
                         exchange=self.px, status=self.bstatus)

    def run_ab(self, l):
        self.run_a(l)
        self.run_b(l)

    def run_c(self):
        self.ver.launch(self.logits, self.ids)

    def run_d(self):
        self.cache.commit(self.new_k, self.new_v, self.ver.result[0], cache_len=self.P)

    def step(self, wait_layer=None, wait_logits=None):
        for l in range(self.L):
            if wait_layer is not None:
                wait_layer(l)
            self.mark("a0")
            self.attention(l, self.q[l], self.kn[l], self.vn[l])
            self.mark("b1")
        self.mark("c0")
        if wait_logits is not None:
            wait_logits()
        self.ver.launch(self.logits, self.ids)
        self.mark("c1")
        self.cache.commit(self.new_k, self.new_v, self.ver.result[0], cache_len=self.P)
        self.mark("d1")

    def statuses(self):
        words = {"a_full": self.plans[False].status, "a_sliding": self.plans[True].status,
                 "b": self.bstatus}
        if self.px is not None:
            words["exchange"] = self.px.status
            words["accept_exchange"] = self.ver.status
        return words

    def close(self):
        if self.px is not None:
            self.px.close()
            self.ver.close()


def bench_cfg5(ctx: Ctx) -> dict:
    import torch
    a = ctx.a
    c = Cfg5(ctx)
    L, N, hq, hk, D, P = c.L, c.N, c.hq, c.hk, c.D, c.P
    before = c.px.reset_stats if c.px is not None else None
    ms_total, clocks, graph = timed_steps(ctx, c.step, a.steps, a.warmup, before)
    del graph
    xwait = c.px.wait_stats() if c.px is not None else None
    k = kernel_ms(ctx, c)
    full = [l for l in range(L) if not c.sliding[l]]
    a_full = graph_ms(ctx, lambda i: c.run_a(full[i % len(full)]), 2 * len(full))
    statuses = check_status(ctx, "config 5", c.statuses())
    hbm, tf_burst, _, peak_src = measured_peaks()
    flops_full = 4.0 * N * hq * P * D
    ach = flops_full / (a_full / 1e3) / 1e12
    bytes_c = c.logits.numel() * 2 + N * 8
    out = {
        "metric": "verified tokens/s", "unit": "tokens/s",
        "value": N * a.steps / (ms_total / 1e3), "ms_per_step": ms_total / a.steps,
        "us_per_layer": (ms_total / a.steps - k["c"] - k["d"]) / L * 1e3,
        "n_gpus": ctx.world, "scaling": "strong",
        "parallelism": (f"kv-head shard x{ctx.world}, output all-gather by kernel (b)'s NVLink "
                        "stores, vocabulary-sharded acceptance" if ctx.world > 1 else "single GPU"),
        "workload": (f"BASELINE config 5: GPT-OSS-20B attention, {L} layers alternating a "
                     f"{c.W}-token sliding window and full attention, {CFG5['qo_heads']}/"
                     f"{CFG5['kv_heads']} heads, D {D}, sinks (reference formula), prefix {P} in "
                     f"16-key UMMA pages, {c.B} x {c.T} tokens, acceptance over [{c.B},{c.T},"
                     f"{c.V}] bf16 logits, commit into {L} layers"),
        "status": statuses, "clocks": clocks,
        "roofline": {"bound": "tensor", "kernel": "prefix_attention_kernel (a) on a full layer "
                     "(D 64)", "achieved": ach, "peak": tf_burst, "unit": "TFLOP/s",
                     "frac": ach / tf_burst,
                     "timing": "kernel (a) back to back over the full layers from a CUDA graph, worst rank",
                     "algorithmic": f"4*N*Hq*P*D = {flops_full:.4g} FLOP per full-layer launch",
                     "peak_source": peak_src},
        "kernels": {"a_full_back_to_back_us": a_full * 1e3, "a_mean_us": k["a"] * 1e3,
                    "b_suffix_merge_sinks_us": k["b"] * 1e3, "b_marginal_us": k["b_marginal"] * 1e3,
                    "c_accept_us": k["c"] * 1e3,
                    "c_accept_gbs": gbs(bytes_c, k["c"]), "d_commit_us": k["d"] * 1e3},
        "gpu_launches": a.steps * (2 * L + 2),
    }
    if xwait is not None:
        out["exchange_wait"] = {"mean_us_per_layer": ctx.max(xwait["mean_wait_us"]),
                                "max_us": ctx.max(xwait["max_wait_us"])}
    if not a.no_e2e:
        out["e2e"] = e2e_static(ctx, c, [c.q, c.kn, c.vn], [c.logits, c.ids],
                                lambda: (c.ver.result, c.ver.accepted), N, "config 5")
    ctx.barrier()
    c.close()
    ctx.barrier()
    del c
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# config 2: Qwen3-8B random init, the full verify forward (1 GPU)
# ---------------------------------------------------------------------------
def qwen3_8b(dev):
    """Qwen3-8B architecture with random weights (std 0.02), bf16, on `dev`."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    c = CFG2
    cfg = Qwen3Config(vocab_size=c["vocab"], hidden_size=c["hidden"],
                      intermediate_size=c["intermediate"], num_hidden_layers=c["layers"],
                      num_attention_heads=c["qo_heads"], num_key_value_heads=c["kv_heads"],
                      head_dim=c["head_dim"], rope_theta=c["rope_theta"], rms_norm_eps=1e-6,
                      max_position_embeddings=40960, tie_word_embeddings=False,
                      initializer_range=0.02)
    cfg._attn_implementation = "sdpa"
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = Qwen3ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    g = torch.Generator(device=dev).manual_seed(2)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=g)
    return model.eval()


def bench_cfg2(ctx: Ctx) -> dict:
    import torch

    import d2sd_b200 as d
    from d2sd_b200.verification import cascade_verify_forward
    a, dev = ctx.a, ctx.dev
    c = CFG2
    B, T, P, V = c["branches"], c["block"], c["prefix"], c["vocab"]
    model = qwen3_8b(dev)
    params = sum(p.numel() * p.element_size() for p in model.parameters())
    g = torch.Generator(device=dev).manual_seed(22)
    with torch.no_grad():
        prefix = torch.randint(0, V, (1, P), generator=g, device=dev)
        cache = model(prefix, use_cache=True).past_key_values
    ids = torch.randint(0, V, (B, T), generator=g, device=dev)
    ids[:, 0] = ids[0, 0]  # the block's anchor token, shared by the branches
    pos = torch.arange(P, P + T, device=dev).view(1, T)
    # drafts of the survey's p = 0.7 draft model: position by position, a
    # branch's token t is the target's argmax at t - 1 with probability 0.7
    # (the forward is causal inside a branch, so fixing t leaves t - 1 as it is)
    with torch.no_grad():
        for t in range(1, T):
            lg, _, _ = cascade_verify_forward(model, ids, pos, cache, True)
            keep = torch.rand(B, generator=g, device=dev) < 0.7
            ids[:, t] = torch.where(keep, lg[:, t - 1].float().argmax(-1), ids[:, t])
    ver = d.BatchVerifier(1, B, T, V, dev)

    def step(_i, input_ids=ids):
        logits, _, _ = cascade_verify_forward(model, input_ids, pos, cache, True)
        ver.launch(logits.view(1, B, T, V), input_ids.view(1, B, T))

    ms_total, clocks, graph = timed_steps(ctx, lambda: step(0), a.steps, a.warmup)
    del graph
    ms = ms_total / a.steps
    acc_len = int(ver.result[0, 0].item())
    # the attention kernels alone on the same shapes (36 x (a)+(b)) for the share
    Hq, Hk, D = c["qo_heads"], c["kv_heads"], c["head_dim"]
    qa = torch.randn(B, T, Hq, D, device=dev, dtype=torch.bfloat16)
    kva = torch.randn(B, T, Hk, D, device=dev, dtype=torch.bfloat16)
    plan = d.CascadePlan([d.Request(B * T, 0, 0, P)], Hq, Hk, D, dev)
    layers = cache.layers
    att_ms = graph_ms(ctx, lambda i: d.cascade_attention(
        qa, kva, kva, layers[i % c["layers"]].keys[0], layers[i % c["layers"]].values[0], "hnd",
        P, plan=plan), c["layers"]) * c["layers"]
    # the reference's own GPU path on the same weights: plain_verify_forward
    # (HF sdpa) branch by branch, cropping the cache back after each branch
    # (generation/verification.py:204-220, generation/d3_generator.py:233-237)
    def hf_step(_i):
        with torch.no_grad():
            for b in range(B):
                model(ids[b:b + 1], position_ids=pos, past_key_values=cache, use_cache=True)
                cache.crop(P)
    hf_ms = ctx.time_ms(hf_step, max(3, a.steps // 4)) / max(3, a.steps // 4)
    hbm, _, _, peak_src = measured_peaks()
    out = {
        "metric": "verified tokens/s", "unit": "tokens/s", "value": B * T / (ms / 1e3),
        "ms_per_step": ms, "n_gpus": 1, "scaling": "strong", "clocks": clocks,
        "committed_tokens_per_s": acc_len / (ms / 1e3), "acceptance_length": acc_len,
        "drafts": "each branch's token t = the target's argmax at t - 1 with probability 0.7",
        "timing": "the step captured once into a CUDA graph and replayed (the HF reference path below runs eagerly, as the reference does)",
        "workload": (f"BASELINE config 2: Qwen3-8B architecture, random init (std 0.02), bf16, "
                     f"{c['layers']} layers, hidden {c['hidden']}, {Hq}/{Hk} heads, D {D}, vocab "
                     f"{V}; prefix {P} random ids (HF prefill into a DynamicCache); one "
                     f"cascade_verify_forward of {B} branches x {T} tokens + acceptance per step"),
        "roofline": {"bound": "hbm (weight reads of the projections, MLP and lm_head)",
                     "achieved": params / (ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": params / (ms / 1e3) / 1e9 / hbm,
                     "algorithmic": f"{params / 1e9:.2f} GB of bf16 weights read per forward",
                     "peak_source": peak_src},
        "attention_share": {"attention_ms": att_ms, "frac_of_step": att_ms / ms,
                            "what": ("36 x kernels (a)+(b) on the forward's shapes, back to back "
                                     "from a CUDA graph")},
        "gpu_reference_hf_sdpa": {"value": B * T / (hf_ms / 1e3), "unit": "tokens/s",
                                  "ms_per_step": hf_ms,
                                  "what": ("the reference's plain_verify_forward (HF sdpa) "
                                           "branch by branch with a cache crop, same GPU and "
                                           "weights")},
        # this library's kernels per step: QK-norm + RoPE, (a) and (b) per layer,
        # then the acceptance (the projections, MLP and lm_head are cuBLAS)
        "gpu_launches": a.steps * (3 * c["layers"] + 1),
    }
    if not a.no_e2e:
        h_ids = ids.cpu().pin_memory()
        d_ids = torch.empty_like(ids)
        h_res = torch.empty(2, dtype=torch.int32).pin_memory()

        def e2e_step(_i):
            d_ids.copy_(h_ids, non_blocking=True)
            step(_i, d_ids)
            h_res.copy_(ver.result[0], non_blocking=True)
            ctx.stream.synchronize()
        for i in range(max(3, a.warmup)):
            e2e_step(i)
        e_ms = ctx.time_ms(e2e_step, a.steps) / a.steps
        out["e2e"] = {"value": B * T / (e_ms / 1e3), "unit": "tokens/s",
                      "h2d_bytes_per_step": h_ids.numel() * 8, "d2h_bytes_per_step": 8,
                      "ms_per_step": e_ms}
    del model, cache
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# config 1: the fp32 single-layer case (1 GPU)
# ---------------------------------------------------------------------------
CFG1 = dict(prefix=512, branches=4, block=16, qo_heads=32, kv_heads=8, head_dim=128, vocab=151936)


def bench_cfg1(ctx: Ctx) -> dict:
    """One fp32 cascade attention layer (d2sd_cascade_attention_f32) and the
    acceptance over fp32 logits: BASELINE config 1 on the GPU."""
    import torch

    import d2sd_b200 as d
    from d2sd_b200 import _lib, ops
    a, dev, c = ctx.a, ctx.dev, CFG1
    P, B, T, Hq, Hk, D, V = (c["prefix"], c["branches"], c["block"], c["qo_heads"],
                             c["kv_heads"], c["head_dim"], c["vocab"])
    g = torch.Generator(device=dev).manual_seed(0)
    r = lambda *sh: torch.randn(*sh, generator=g, device=dev) / D ** 0.5  # noqa: E731
    q, kn, vn, kp, vp = r(B * T, Hq, D), r(B * T, Hk, D), r(B * T, Hk, D), r(P, Hk, D), r(P, Hk, D)
    logits = torch.randn(1, B, T, V, generator=g, device=dev)
    ids = torch.randint(0, V, (1, B, T), generator=g, device=dev)
    keep = torch.rand(1, B, T, generator=g, device=dev) < 0.7
    ids[..., 1:] = torch.where(keep[..., 1:], logits.argmax(-1)[..., :-1], ids[..., 1:])
    ids[..., 0] = ids[0, 0, 0]
    out = torch.empty(B * T, Hq, D, device=dev)
    lse = torch.empty(B * T, Hq, device=dev)
    ver = d.BatchVerifier(1, B, T, V, dev)

    def attn():
        ops.cascade_attention_f32(q, out, lse, num_blocks=B, block_len=T, num_kv_heads=Hk,
                                  sm_scale=D ** -0.5, k_prefix=kp, v_prefix=vp, k_local=kn,
                                  v_local=vn, mask_mode=_lib.MASK_CAUSAL)

    def step():
        attn()
        ver.launch(logits, ids)

    ms_total, clocks, graph = timed_steps(ctx, step, a.steps, a.warmup)
    del graph
    att = graph_ms(ctx, lambda i: attn(), 10)
    acc = graph_ms(ctx, lambda i: ver.launch(logits, ids), 10)
    hbm, _, _, peak_src = measured_peaks()
    out_d = {"metric": "verified tokens/s", "unit": "tokens/s", "value": B * T * a.steps / (ms_total / 1e3),
             "ms_per_step": ms_total / a.steps, "n_gpus": 1, "scaling": "strong", "dtype": "f32",
             "clocks": clocks,
             "workload": (f"BASELINE config 1: fp32, seed 0, prefix {P}, {Hq}/{Hk} heads, D {D}, "
                          f"{B} x {T} tokens causal in each branch, one layer of the fp32 cascade "
                          f"(d2sd_cascade_attention_f32) + acceptance over [{B},{T},{V}] fp32 logits"),
             "kernels": {"attention_f32_us": att * 1e3, "accept_us": acc * 1e3,
                         "accept_gbs": gbs(logits.numel() * 4, acc)},
             "roofline": {"bound": "hbm (acceptance: fp32 logits read once)", "kernel": "accept_kernel",
                          "achieved": gbs(logits.numel() * 4, acc), "peak": hbm, "unit": "GB/s",
                          "frac": gbs(logits.numel() * 4, acc) / hbm, "peak_source": peak_src},
             "tolerance": "1e-5 abs/rel against the float64 oracle (tests/test_fp32_gpu.py)",
             "gpu_launches": a.steps * 2}
    if not a.no_e2e:
        h_in = [t.cpu().pin_memory() for t in (q, kn, vn, kp, vp, logits, ids)]
        d_in = (q, kn, vn, kp, vp, logits, ids)
        h_res = torch.empty(2, dtype=torch.int32).pin_memory()

        def e2e_step(_i):
            for dt, ht in zip(d_in, h_in):
                dt.copy_(ht, non_blocking=True)
            step()
            h_res.copy_(ver.result[0], non_blocking=True)
            ctx.stream.synchronize()
        for i in range(max(3, a.warmup)):
            e2e_step(i)
        e_ms = ctx.time_ms(e2e_step, a.steps) / a.steps
        out_d["e2e"] = {"value": B * T / (e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in h_in),
                        "d2h_bytes_per_step": 8, "ms_per_step": e_ms}
    return out_d


def cpu_cfg1(reps: int = 5) -> dict:
    """Config 1 on the CPU: the fp32 tree-masked torch.sdpa layer and the walk."""
    import numpy as np
    import torch

    from oracle import accept as OA
    from oracle import attention as AT
    cores = cpu_threads()
    c = CFG1
    P, B, T, Hq, Hk, D, V = (c["prefix"], c["branches"], c["block"], c["qo_heads"],
                             c["kv_heads"], c["head_dim"], c["vocab"])
    g = torch.Generator().manual_seed(0)
    r = lambda *sh: torch.randn(*sh, generator=g) / D ** 0.5  # noqa: E731
    q, kn, vn, kp, vp = r(B, T, Hq, D), r(B, T, Hk, D), r(B, T, Hk, D), r(P, Hk, D), r(P, Hk, D)
    z = torch.randn(B, T, V, generator=g).numpy()
    x = np.random.default_rng(0).integers(0, V, (B, T))
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        AT.torch_tree_sdpa(q, kn, vn, kp, vp, causal=True)
        OA.verify_accept(z, x)
        ts.append(time.perf_counter() - t0)
    step = statistics.median(ts)
    return {"value": B * T / step, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"median of {reps} x [one fp32 tree-masked torch.sdpa layer (P {P}, "
                       f"{B} x {T} tokens, {Hq}/{Hk} heads, D {D}) + the acceptance walk over "
                       f"[{B},{T},{V}] fp32 logits] = one step"),
            "seconds_per_step": step}


# ---------------------------------------------------------------------------
# the d2sd arm
# ---------------------------------------------------------------------------
def run_d2sd(ctx: Ctx):
    a, world, rank = ctx.a, ctx.world, ctx.rank
    which = [x.strip() for x in a.configs.split(",") if x.strip()]
    cpu = rank == 0 and world == 1 and not a.no_cpu_baseline
    subs = {}

    def sub(name, fn, cpu_fn):
        if world == 1:
            try:  # one GPU: a failing sub-config is reported, the headline still prints
                subs[name] = fn(ctx)
            except Exception as e:  # noqa: BLE001
                subs[name] = {"error": f"{type(e).__name__}: {e}"}
                return
        else:
            subs[name] = fn(ctx)
        if cpu and cpu_fn is not None:
            cb = cpu_fn()
            cb.pop("seconds_per_step", None)
            subs[name]["cpu_baseline"] = cb

    head = bench_cfg3(ctx) if "3" in which else None
    if "3" in which and world == 1 and not a.shared:
        for k in (4, 8):  # config 3's tree-trunk sweep
            sub(f"cfg3_trunk{k}", lambda cx, k=k: bench_cfg3_trunk(cx, k), None)
    if "4" in which:
        sub("cfg4", bench_cfg4, cpu_cfg4)
    if "5" in which:
        sub("cfg5", bench_cfg5, cpu_cfg5)
    if "1" in which:
        if world == 1:
            sub("cfg1", bench_cfg1, cpu_cfg1)
        else:
            subs["cfg1"] = {"skipped": "config 1 is a one-GPU configuration"}
    if "2" in which:
        if world == 1:
            sub("cfg2", bench_cfg2, cpu_cfg2)
        else:
            subs["cfg2"] = {"skipped": "config 2 is a one-GPU configuration"}
    if head is None:
        if rank == 0:
            print(json.dumps({"configs": subs}), flush=True)
        return
    line = {
        "metric": "verified tokens/s", "value": head["value"], "unit": "tokens/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V and logits; drafts match argmax w.p. 0.7)",
        "config": workload_config(a, world),
    }
    line.update({k: v for k, v in head.items() if k not in ("value", "ms_per_step")})
    if cpu:
        cb = cpu_cfg3(a)
        cb.pop("seconds_per_step", None)
        line["cpu_baseline"] = cb
    line["configs"] = subs
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local_rank}"))
    try:
        run_d2sd(Ctx(a, rank, world, local_rank))
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
