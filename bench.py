"""Benchmark of the D2-SD verify hot path on B200.

Default workload (the north-star shape, on Qwen3-8B's 36
layers): one verify step of one request = for every layer, the two-level
cascade attention of 8 branches x 32 block tokens over a 32768-token paged
prefix (kernel a: shared prefix on tcgen05/TMEM, kernel b: per-branch causal
suffix fused with the LSE merge), then greedy acceptance over the bf16 target
logits [8, 32, 151936] (kernel c), then the commit of the accepted rows into
all 36 layers' paged caches (kernel d). A step verifies B*T = 256 candidate
tokens; the metric is verified tokens/s (B*T / step time). The commit writes
the same cache slots every step so every step does identical work.

Multi-GPU (torchrun, one rank per GPU): KV-head sharding (strong scaling) --
rank r owns Hk/N kv heads of every layer and their pages, runs kernels a+b on
them, and NCCL all-gathers the attention output of each layer; acceptance runs
on every rank over the replicated logits, the commit on the local heads.

--impl reference: the reference's own CPU path (torch.sdpa masked attention +
the acceptance walk + the cat-based commit, as restated in oracle/) on the
host cores, on a bounded sample of the same step, extrapolated to the step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

# the default workload (BASELINE config 3 on Qwen3-8B heads)
CFG = dict(layers=36, prefix=32768, branches=8, block=32, qo_heads=32, kv_heads=8, head_dim=128,
           vocab=151936, page_size=16, shared=0)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["d2sd", "reference"], default="d2sd")
    ap.add_argument("--layers", type=int, default=CFG["layers"])
    ap.add_argument("--prefix", type=int, default=CFG["prefix"])
    ap.add_argument("--branches", type=int, default=CFG["branches"])
    ap.add_argument("--block", type=int, default=CFG["block"])
    ap.add_argument("--shared", type=int, default=CFG["shared"],
                    help="tokens every branch shares (tree trunk); 0 = independent branches")
    ap.add_argument("--kv-layout", choices=["umma", "hnd"], default="umma",
                    help="page format of the target cache (tensor-core order or plain rows)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="multi-GPU output all-gather: kernel (b)'s own NVLink stores, or NCCL")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def workload_config(a, n):
    return {
        "workload": (f"BASELINE config 3 verify step on Qwen3-8B heads: {a.layers} layers x "
                     f"cascade attention ({CFG['qo_heads']}q/{CFG['kv_heads']}kv heads, D "
                     f"{CFG['head_dim']}, prefix {a.prefix} paged (page {CFG['page_size']}), "
                     f"{a.branches} branches x {a.block} tokens, tree trunk k={a.shared}) + greedy "
                     f"acceptance over [{a.branches},{a.block},{CFG['vocab']}] bf16 logits + KV "
                     f"commit into {a.layers} layers"),
        "global_batch": a.branches * a.block,
        "seq_len": a.prefix,
        "parallelism": (f"kv-head shard x{n}, per-layer output all-gather "
                        + ("by kernel (b)'s NVLink stores" if a.exchange == "peer" else "by NCCL")
                        if n > 1 else "single GPU"),
        "l2": "inputs larger than L2 (paged KV of all layers streamed each step)",
        "kv_pages": ("16-key pages in tensor-core core-matrix order" if a.kv_layout == "umma"
                     else "16-key pages of plain rows [page, head, slot, dim]"),
    }


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
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


def profile_traffic(name: str):
    """dram bytes per launch of kernel (a) from the committed ncu summary."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU path, restated in oracle/)
# ---------------------------------------------------------------------------
def cpu_sample(a, budget_s: float = 12.0):
    """Time the reference CPU path on a bounded sample: one branch of one layer
    of the attention (torch.sdpa masked + logsumexp), the acceptance walk over
    the full logits, and the commit; extrapolate to the whole step."""
    import numpy as np
    import torch

    from oracle import accept as OA
    from oracle import attention as AT
    from oracle import commit as OC
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)
    Hq, Hk, D, P, T, B = CFG["qo_heads"], CFG["kv_heads"], CFG["head_dim"], a.prefix, a.block, a.branches
    q = torch.randn(1, T, Hq, D, generator=g)
    kn = torch.randn(1, T, Hk, D, generator=g)
    vn = torch.randn(1, T, Hk, D, generator=g)
    kp = torch.randn(P, Hk, D, generator=g)
    vp = torch.randn(P, Hk, D, generator=g)
    z = torch.randn(B, T, CFG["vocab"], generator=g)
    x = torch.randint(0, CFG["vocab"], (B, T), generator=g)
    x[:, 1:] = torch.where(torch.rand(B, T - 1, generator=g) < 0.7, z.argmax(-1)[:, :-1], x[:, 1:])
    zn, xn = z.numpy(), x.numpy()
    cache_k = [np.zeros((1, Hk, P, D), np.float32) for _ in range(2)]
    new = [(np.random.default_rng(1).standard_normal((B, Hk, T, D)).astype(np.float32),) * 2
           for _ in range(2)]
    t_att, t_acc, t_com = [], [], []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        AT.torch_masked_sdpa(q, kn, vn, kp, vp, causal=True)
        t1 = time.perf_counter()
        acc, _, br = OA.verify_accept(zn, xn)
        t2 = time.perf_counter()
        OC.commit_contiguous(cache_k, cache_k, new, br, acc)  # 2 of the layers
        t3 = time.perf_counter()
        t_att.append(t1 - t0)
        t_acc.append(t2 - t1)
        t_com.append((t3 - t2) / 2)
        if time.perf_counter() - t_start > budget_s or len(t_att) >= 5:
            break
    att, acc_t, com = (statistics.median(v) for v in (t_att, t_acc, t_com))
    step = a.layers * B * att + acc_t + a.layers * com
    return {
        "value": B * T / step,
        "unit": "tokens/s",
        "cores": cores,
        "kind": "port",
        "sample": (f"{len(t_att)}x [one branch of one layer of the fp32 torch.sdpa masked attention "
                   f"(P={P}, {T} tokens, {Hq}/{Hk} heads, D={D}) + the acceptance walk over "
                   f"[{B},{T},{CFG['vocab']}] fp32 logits + the cat commit of 2 layers], median, "
                   f"extrapolated to {a.layers} layers x {B} branches"),
        "seconds_per_step": step,
    }


def run_reference(a, rank: int, world: int):
    if rank != 0:
        return
    K, W = a.steps, a.warmup
    # each step: one bounded sample (see cpu_sample); warm-up steps untimed
    for _ in range(max(0, W)):
        cpu_sample(a, budget_s=0.0)
    vals = []
    t0 = time.perf_counter()
    res = None
    for _ in range(K):
        res = cpu_sample(a, budget_s=0.0)
        vals.append(res["seconds_per_step"])
    wall = time.perf_counter() - t0
    step = statistics.median(vals)
    value = a.branches * a.block / step
    line = {
        "impl": "reference", "metric": "verified tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(a, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": res["cores"],
                         "kind": "port", "sample": res["sample"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "wall_s": wall,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the d2sd arm
# ---------------------------------------------------------------------------
def run_d2sd(a, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    import d2sd_b200 as d
    from d2sd_b200 import ops

    dev = torch.device(f"cuda:{local_rank}")
    torch.cuda.set_device(dev)
    L, P, B, T = a.layers, a.prefix, a.branches, a.block
    Hq, Hk, D, V = CFG["qo_heads"], CFG["kv_heads"], CFG["head_dim"], CFG["vocab"]
    if Hk % world:
        raise SystemExit(f"{Hk} kv heads do not shard over {world} GPUs")
    hk, hq = Hk // world, Hq // world
    N = B * T
    n_u = a.shared + B * (T - a.shared) if a.shared else N
    scale = D ** -0.5
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    # --- state resident in HBM -------------------------------------------
    cache = d.PagedKVCache(L, hk, D, P + T + 16, device=dev, layout=a.kv_layout,
                           page_order=torch.randperm(-(-(P + T + 16) // 16),
                                                     generator=torch.Generator().manual_seed(7)))
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    cache.length = P
    q = torch.randn(L, B, T, hq, D, generator=g, device=dev).to(torch.bfloat16)
    if a.shared:
        q[:, :, :a.shared] = q[:, 0:1, :a.shared]
    kn = torch.randn(L, B, T, hk, D, generator=g, device=dev).to(torch.bfloat16)
    vn = torch.randn(L, B, T, hk, D, generator=g, device=dev).to(torch.bfloat16)
    gz = torch.Generator(device=dev).manual_seed(99)  # logits replicated on every rank
    logits = torch.randn(B, T, V, generator=gz, device=dev).to(torch.bfloat16)
    ids = torch.randint(0, V, (B, T), generator=gz, device=dev)
    keep = torch.rand(B, T, generator=gz, device=dev) < 0.7
    ids[:, 1:] = torch.where(keep[:, 1:], logits.float().argmax(-1)[:, :-1], ids[:, 1:])
    ids[:, 0] = ids[0, 0]

    plan = d.CascadePlan([d.Request(n_u, 0, 0, P)], hq, hk, D, dev)
    ptok = d.shared_trunk_map(B, T, a.shared, dev) if a.shared else None
    q_pref = [torch.cat([q[l, 0, :a.shared], q[l, :, a.shared:].reshape(-1, hq, D)], 0)
              if a.shared else q[l].reshape(N, hq, D) for l in range(L)]
    out = torch.empty(N, hq, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(N, hq, dtype=torch.float32, device=dev)
    gathered = (torch.empty(world * N, hq, D, dtype=torch.bfloat16, device=dev)
                if world > 1 and a.exchange == "nccl" else None)
    px = (d.PeerExchange(N, Hq, Hk, D, torch.bfloat16, dev)
          if world > 1 and a.exchange == "peer" else None)
    ver = d.Verifier(B, T, V, dev)
    new_k = kn.transpose(2, 3)  # [L, B, hk, T, D] views of the token-major K/V
    new_v = vn.transpose(2, 3)
    stream = torch.cuda.current_stream(dev)

    ev = {}

    def mark(name):
        if ev is not None and name in ev:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            ev[name].append(e)

    bstatus = torch.zeros(1, dtype=torch.int32, device=dev)  # kernel (b)'s wait time-outs

    def step(qs, kns, vns, lg, bid, timing=False, wait_layer=None, wait_logits=None):
        for l in range(L):
            if wait_layer is not None:
                wait_layer(l)
            if timing:
                mark("a0")
            plan.run_prefix(qs[l], cache.k[l], cache.v[l], cache.kv_layout, scale,
                            page_table=cache.page_table)
            if timing:
                mark("a1")
            ops.suffix_merge(qs_full[l], kns[l].reshape(N, hk, D), vns[l].reshape(N, hk, D), out,
                             lse, num_blocks=B, block_len=T, num_qo_heads=hq, num_kv_heads=hk,
                             sm_scale=scale, partial=plan.partial, plan_dev=plan.plan,
                             prefix_token=ptok, exchange=px, status=bstatus)
            if timing:
                mark("b1")
            if gathered is not None:
                dist.all_gather_into_tensor(gathered, out)
        if timing:
            mark("c0")
        if wait_logits is not None:
            wait_logits()
        ver.launch(lg, bid)
        if timing:
            mark("c1")
        cache.commit(new_k, new_v, ver.result, cache_len=P)
        if timing:
            mark("d1")

    qs_full = [q[l].reshape(N, hq, D) for l in range(L)]
    kns = [kn[l] for l in range(L)]
    vns = [vn[l] for l in range(L)]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # --- device-resident timing ----------------------------------------------
    for _ in range(max(3, a.warmup)):
        step(q_pref, kns, vns, logits, ids)
    barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    ev = {k: [] for k in ("a0", "a1", "b1", "c0", "c1", "d1")}
    if px is not None:
        px.reset_stats()
    barrier()
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_begin.record(stream)
    for i in range(a.steps):
        step(q_pref, kns, vns, logits, ids)
    t_end.record(stream)
    barrier()
    clocks = sampler.stop()
    ms_total = max_over_ranks(t_begin.elapsed_time(t_end))
    ms_step = ms_total / a.steps
    xwait = px.wait_stats() if px is not None else None
    # per-kernel events on one extra step after the timed region: an event
    # between two kernels keeps the second from starting early (the programmatic
    # launch overlap), so a marked step runs slower than the timed ones; it
    # gives one event pair per launch of (a) and (b) for every layer
    step(q_pref, kns, vns, logits, ids, timing=True)
    barrier()
    a_ms = [s.elapsed_time(e) for s, e in zip(ev["a0"], ev["a1"])]
    b_ms = [s.elapsed_time(e) for s, e in zip(ev["a1"], ev["b1"])]
    c_ms = [s.elapsed_time(e) for s, e in zip(ev["c0"], ev["c1"])]
    d_ms = [s.elapsed_time(e) for s, e in zip(ev["c1"], ev["d1"])]
    a_avg = max_over_ranks(statistics.mean(a_ms))
    b_avg = max_over_ranks(statistics.mean(b_ms))
    c_avg = max_over_ranks(statistics.mean(c_ms))
    d_avg = max_over_ranks(statistics.mean(d_ms))
    acc_len = int(ver.result[0].item())

    # --- back-to-back kernel timing (after the timed region) ------------------
    # An event between two kernels stops the second from starting early, so the
    # per-kernel events above include each launch's latency. Here kernel (a)
    # runs alone over all layers twice, then (a)+(b): no events in between, the
    # programmatic launch overlap intact.
    def loop_ms(fn, reps: int = 2) -> float:
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            for l in range(L):
                fn(l)
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / (reps * L)

    def run_a(l):
        plan.run_prefix(q_pref[l], cache.k[l], cache.v[l], cache.kv_layout, scale,
                        page_table=cache.page_table)

    def run_ab(l):
        run_a(l)
        ops.suffix_merge(qs_full[l], kns[l].reshape(N, hk, D), vns[l].reshape(N, hk, D), out, lse,
                         num_blocks=B, block_len=T, num_qo_heads=hq, num_kv_heads=hk,
                         sm_scale=scale, partial=plan.partial, plan_dev=plan.plan,
                         prefix_token=ptok, exchange=px)
        if gathered is not None:
            dist.all_gather_into_tensor(gathered, out)

    a_b2b = loop_ms(run_a)
    ab_b2b = loop_ms(run_ab)
    value = N * a.steps / (ms_total / 1e3)
    # no line from a run in which any kernel gave up a bounded wait
    statuses = {"a": int(plan.status.item()), "b": int(bstatus.item())}
    if px is not None:
        statuses["exchange"] = int(px.status.item())
    bad = {k: v for k, v in statuses.items() if v}
    if bad:
        raise SystemExit(f"rank {rank}: kernel status words nonzero {bad}: no bench line")

    # --- end to end: host buffers, copies inside the timed region --------------
    e2e = None
    if not a.no_e2e:
        pin = lambda t: t.cpu().pin_memory()  # noqa: E731
        hq_pref = [pin(t) for t in q_pref]
        hq_full = [pin(t) for t in qs_full]
        hkn = [pin(t) for t in kns]
        hvn = [pin(t) for t in vns]
        h_logits = pin(logits)
        h_ids = pin(ids)
        d_qp = [torch.empty_like(t) for t in q_pref]
        d_qf = [torch.empty_like(t) for t in qs_full]
        d_kn = [torch.empty_like(t) for t in kns]
        d_vn = [torch.empty_like(t) for t in vns]
        d_logits = torch.empty_like(logits)
        d_ids = torch.empty_like(ids)
        h_res = torch.empty(2, dtype=torch.int32).pin_memory()
        h_acc = torch.empty(T, dtype=torch.int64).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in hq_pref + hkn + hvn + [h_logits, h_ids])
        if a.shared:
            h2d += sum(t.numel() * t.element_size() for t in hq_full)
        d2h = h_res.numel() * 4 + h_acc.numel() * 8

        # host->device copies run on their own stream, layer by layer, and
        # layer l's attention waits only for layer l's inputs: the copies of
        # later layers (and of the logits) overlap the attention of earlier ones
        copy_stream = torch.cuda.Stream(dev)
        ev_layer = [torch.cuda.Event() for _ in range(L)]
        ev_logits = torch.cuda.Event()

        def e2e_step():
            copy_stream.wait_stream(stream)  # after the timer start and the previous step
            with torch.cuda.stream(copy_stream):
                for l in range(L):
                    d_qp[l].copy_(hq_pref[l], non_blocking=True)
                    if a.shared:
                        d_qf[l].copy_(hq_full[l], non_blocking=True)
                    d_kn[l].copy_(hkn[l], non_blocking=True)
                    d_vn[l].copy_(hvn[l], non_blocking=True)
                    ev_layer[l].record(copy_stream)
                d_logits.copy_(h_logits, non_blocking=True)
                d_ids.copy_(h_ids, non_blocking=True)
                ev_logits.record(copy_stream)
            nonlocal qs_full
            saved = qs_full
            if a.shared:
                qs_full = d_qf
            else:
                qs_full = [t.view(N, hq, D) for t in d_qp]
            step(d_qp, d_kn, d_vn, d_logits, d_ids,
                 wait_layer=lambda l: stream.wait_event(ev_layer[l]),
                 wait_logits=lambda: stream.wait_event(ev_logits))
            qs_full = saved
            h_res.copy_(ver.result, non_blocking=True)
            h_acc.copy_(ver.accepted, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        for _ in range(max(3, a.warmup)):
            e2e_step()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            e2e_step()
        e1.record(stream)
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": N * a.steps / (e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms / a.steps}

    # --- roofline of kernel (a) ---------------------------------------------
    hbm, tf_burst, tf_sust, peak_src = measured_peaks()
    flops_a = 4.0 * n_u * hq * P * D
    achieved = flops_a / (a_avg / 1e3) / 1e12
    traffic = profile_traffic("prefix_attention_cfg3.txt") if (world == 1 and P == 32768 and
                                                                not a.shared) else None
    achieved_b2b = flops_a / (a_b2b / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
                "frac": achieved / tf_burst, "traffic": traffic,
                "achieved_back_to_back": achieved_b2b, "frac_back_to_back": achieved_b2b / tf_burst,
                "frac_of_sustained": achieved / tf_sust,
                "timing": ("achieved: per-launch CUDA events on a marked step after the timed "
                           "region (each includes its launch latency); back_to_back: kernel (a) "
                           "alone over all layers, events around the loop only"),
                "peak_source": (f"bf16_tflops (burst) of {peak_src}: the timed region lasts "
                                f"{ms_total / 1e3:.2f} s at full clock"),
                "kernel": "prefix_attention_kernel (a)",
                "algorithmic": f"4*N_u*Hq*P*D = {flops_a:.4g} FLOP per launch"}
    bytes_c = B * T * V * 2 + B * T * 8
    kv_bytes_a = 2 * P * hk * D * 2
    # kernel (b): Q, the block's K/V, O, LSE, plus the partial slots it merges
    slot_b = (plan.partial.numel() * plan.partial.element_size()) if plan.partial is not None else 0
    bytes_b = N * hq * D * 2 + 2 * N * hk * D * 2 + N * hq * D * 2 + N * hq * 4 + slot_b
    bytes_d = 2 * acc_len * L * 2 * hk * D * 2
    gbs = lambda nbytes, ms: nbytes / (ms / 1e3) / 1e9  # noqa: E731
    kernels = {
        "a_prefix_attention_us": a_avg * 1e3,
        "a_hbm_floor_us": kv_bytes_a / (hbm * 1e9) * 1e6,
        "b_suffix_merge_us": b_avg * 1e3,
        "b_suffix_merge_gbs": gbs(bytes_b, b_avg),
        "c_accept_us": c_avg * 1e3,
        "c_accept_gbs": gbs(bytes_c, c_avg),
        "d_commit_us": d_avg * 1e3,
        "d_commit_gbs": gbs(bytes_d, d_avg),
        "hbm_peak_gbs": hbm,
        "hbm_frac": {"b": gbs(bytes_b, b_avg) / hbm, "c": gbs(bytes_c, c_avg) / hbm,
                     "d": gbs(bytes_d, d_avg) / hbm},
        "attention_us_per_layer_marked": (a_avg + b_avg) * 1e3,
        "a_back_to_back_us": a_b2b * 1e3,
        "b_marginal_back_to_back_us": (ab_b2b - a_b2b) * 1e3,
        "acceptance_length": acc_len,
    }
    line = {
        "metric": "verified tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V and logits; drafts match argmax w.p. 0.7)",
        "config": workload_config(a, world),
        "us_per_layer": (ms_step - c_avg - d_avg) / L * 1e3,
        "status": statuses,
        "roofline": roofline, "kernels": kernels, "clocks": clocks, "e2e": e2e,
        "gpu_launches": a.steps * (2 * L + 2),
    }
    if xwait is not None:
        # time the signalling CTA of kernel (b) waited for the other ranks, per
        # layer, in the timed region (the worst rank's mean and maximum)
        line["exchange_wait"] = {"mean_us_per_layer": max_over_ranks(xwait["mean_wait_us"]),
                                 "max_us": max_over_ranks(xwait["max_wait_us"]),
                                 "waits": xwait["waits"]}
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cb = cpu_sample(a)
        cb.pop("seconds_per_step", None)
        line["cpu_baseline"] = cb
    if rank == 0:
        print(json.dumps(line), flush=True)
    if px is not None:
        barrier()  # every rank's kernels are done with the peers' buffers
        px.close()


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
        run_d2sd(a, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
