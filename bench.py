"""Benchmark: paged decode attention HBM GB/s (and decode tokens/s) on B200.

Default workload (N=1): INT8 paged decode attention at the GPT-2-small shape,
batch 32, 12 heads (MHA), head_dim 64, block_size 16, every context ~1024,
fp16 K/V/Q ~ N(0,1), physical pages shuffled by the allocator.  One step is a
decode step over 12 layers (GPT-2 small depth, one pool per layer): one
allocator/planner launch, then per layer the KV append of one new token per
sequence (a page commit every 16 steps) and the fused attention.  The 12
pools (~610 MB) exceed the 126 MB L2, so no flush is needed between steps.

The step runs as one CUDA graph (metagross_b200.DecodeGraph: begin_step, the
step's decode plan, then per layer append + attention), so it is bound by the
GPU rather than by per-kernel launch cost; sequence truncation stays an eager
cache call.  The attention kernel's own time is measured on a graph of the 12
attention launches alone (CUDA events around the replays).

Each sequence's context stays within one page of its configured length: it
grows one token per step and every 16 steps its last page is truncated back
to the allocator (a real cache operation, counted in the timed region), so
the timed steps see contexts 1009..1024 (mean ~1016.5) with one page commit
per sequence every 16 steps (at context 1024).

Metric value = algorithmic HBM bytes of the step (codes, scales, block table,
staged tail, q, out, append traffic; each byte counted once) / device time.
With --gpus N (torchrun) every rank runs the same per-GPU workload on its own
sequences (weak scaling) and the last layer's outputs are gathered with NCCL
all_gather once per step; time is the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gpt2_int8|tinyllama_int4]
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

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # config: INT8 MHA, GPT-2 small
    "gpt2_int8": dict(batch=32, hq=12, hkv=12, d=64, page=16, ctx=1024, layers=12, kv="int8",
                      desc="INT8 paged decode attention, GPT-2-small shape: batch 32, 12 heads, head_dim 64, "
                           "block 16, context 1024, 12 layers, 1 new token/seq/step"),
    # config: INT4 GQA, TinyLlama attention shape, contexts U[128, 2048], 1% outliers x8
    "tinyllama_int4": dict(batch=64, hq=32, hkv=4, d=64, page=16, ctx="uniform128_2048", layers=22, kv="int4",
                           desc="INT4 paged decode attention with GQA (32q/4kv), head_dim 64, block 16, batch 64, "
                                "contexts U[128,2048], 22 layers, 1% outliers x8"),
    # config: 1024 sequences sharded over the GPUs (strong scaling), log-normal contexts
    "lognormal_int4": dict(batch=1024, hq=32, hkv=4, d=64, page=16, ctx="lognormal2048", layers=4, kv="int4",
                           sharded=True,
                           desc="INT4 paged decode attention, TinyLlama attention shape (32q/4kv, head_dim 64, "
                                "block 16), 1024 sequences with contexts exp(N(ln 2048, 1.0)) capped at 32768, "
                                "sharded over the GPUs by LPT on context length, 4 layers (pools > L2)"),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# --------------------------------------------------------------------------
# algorithmic bytes (counted once per byte that must move)
# --------------------------------------------------------------------------

def attention_bytes(lens, w):
    """Bytes one attention launch must touch: committed codes K+V, per-page scales
    K+V, block-table entries, staged fp16 tail K+V, q and out (fp16)."""
    bq = 1.0 if w["kv"] == "int8" else 0.5
    P, hkv, d, hq = w["page"], w["hkv"], w["d"], w["hq"]
    tot = 0.0
    for c in lens:
        n, r = c // P, c % P
        tot += 2 * n * P * hkv * d * bq + 2 * 4 * n + 4 * n + 2 * 2 * r * hkv * d + 2 * 2 * hq * d
    return tot


def append_bytes(lens_after, w):
    """One new token per sequence: read it (K+V fp16); a filling page also reads
    its P-1 staged rows and writes P rows of codes + 2 scales, otherwise the
    token is written to staging."""
    bq = 1.0 if w["kv"] == "int8" else 0.5
    P, hkv, d = w["page"], w["hkv"], w["d"]
    row = hkv * d
    tot = 0.0
    for c in lens_after:
        tot += 2 * row * 2
        if c % P == 0:
            tot += 2 * (P - 1) * row * 2 + 2 * P * row * bq + 8
        else:
            tot += 2 * row * 2
    return tot


def append_sweep_bytes(old_lens, new_lens, w):
    """Bytes one append launch must move for a step of any size: the new tokens
    (K+V fp16) read once; every page that fills writes its codes (K+V) and two
    scales and reads the rows it had staged before the step; the step's tokens of
    the page left partial are written to staging."""
    bq = 1.0 if w["kv"] == "int8" else 0.5
    P, row = w["page"], w["hkv"] * w["d"]
    tot = 0.0
    for o, n in zip(old_lens, new_lens):
        commits = n // P - o // P
        tot += 2 * (n - o) * row * 2
        if commits > 0:
            tot += commits * (2 * P * row * bq + 8) + 2 * (o % P) * row * 2
        tot += 2 * (n - max(o, (n // P) * P)) * row * 2
    return tot


# --------------------------------------------------------------------------
# clocks sampling during the timed region
# --------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and throttle reasons with nvidia-smi every 50 ms while
    the timed region runs (line-buffered through stdbuf; rows are kept only
    between mark_start() and mark_stop())."""

    FIELDS = ("timestamp,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device_index):
        self.proc = None
        self.rows = []
        self.window = [None, None]
        try:
            p = torch.cuda.get_device_properties(device_index)
            self.bus = f"{p.pci_bus_id:02x}:{p.pci_device_id:02x}".lower()
        except Exception:
            self.bus = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        try:
            self.proc = subprocess.Popen(["stdbuf", "-oL"] + cmd, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()
        time.sleep(0.3)  # first samples arrive before the timed region starts

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), line.strip()))

    def mark_start(self):
        self.window[0] = time.time()

    def mark_stop(self):
        self.window[1] = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        t0, t1 = self.window
        sm, smax, reasons, power = [], None, set(), []
        for ts, ln in self.rows:
            if t0 is not None and not (t0 - 0.06 <= ts <= (t1 or ts) + 0.06):
                continue
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            if self.bus and self.bus not in parts[1].lower():
                continue
            try:
                sm.append(float(parts[2]))
                smax = float(parts[3])
                power.append(float(parts[4]))
            except ValueError:
                continue
            for n, v in zip(self.NAMES, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_median": statistics.median(power) if power else None}


# --------------------------------------------------------------------------
# workload construction
# --------------------------------------------------------------------------

def contexts_for(w, batch, seed):
    g = torch.Generator().manual_seed(seed)
    if w["ctx"] == "uniform128_2048":
        c = torch.randint(128, 2049, (batch,), generator=g)
    elif w["ctx"] == "lognormal2048":
        r = np.random.default_rng(seed)
        c = torch.from_numpy(np.exp(r.normal(np.log(2048.0), 1.0, batch)).round().clip(1, 32768).astype(np.int64))
    else:
        c = torch.full((batch,), int(w["ctx"]))
    return c.to(torch.int32)


class Schedule:
    """Host shadow of the per-sequence lengths.  Sequence b oscillates in
    (base_b, base_b + P]: it grows by one token per step and, once it reaches
    base_b + P, is truncated back to the page boundary base_b (its last page
    returns to the allocator) before the next step.  base_b = floor((c_b-1)/P)*P
    for the workload's context c_b, so contexts stay within one page of c_b
    and every sequence commits one page every P steps."""

    def __init__(self, ctx, P):
        self.P = P
        self.base = ((ctx - 1) // P) * P
        self.cur = ctx - 1  # prefilled length; the first step appends token c_b

    def next_step(self):
        """(truncate ids or None, new lens or None, lengths after the step)"""
        hit = self.cur >= self.base + self.P
        ids = lens = None
        if bool(hit.any()):
            ids = torch.nonzero(hit).flatten().to(torch.int32)
            lens = self.base[hit].to(torch.int32)
            self.cur = torch.where(hit, self.base, self.cur)
        self.cur = self.cur + 1
        return ids, lens, self.cur.clone()


def build(w, device, seed, ctx=None):
    from metagross_b200.batched import BatchedPagedKVCache

    L, hkv, d, P, hq = w["layers"], w["hkv"], w["d"], w["page"], w["hq"]
    if ctx is None:
        ctx = contexts_for(w, w["batch"], seed)
    B = int(ctx.numel())
    start = ctx - 1
    max_final = int(ctx.max()) + P
    max_blocks = max_final // P + 2
    # pool with slack so physical pages come out of a shuffled free list
    num_pages = int(((ctx.to(torch.int64) + 2 * P - 1) // P + 1).sum()) + 256
    cache = BatchedPagedKVCache(L, B, hkv, d, page_size=P, num_pages=num_pages, max_blocks=max_blocks,
                                kv_dtype=w["kv"], staging_dtype=torch.float16, device=device)
    cache._workspace(hq, max_final)  # size the split workspace once, outside any timed region
    # shuffle the allocator's free stack so logical pages land on random physical pages
    g = torch.Generator().manual_seed(seed + 1)
    perm = torch.randperm(num_pages, generator=g).to(torch.int32)
    cache.allocator.free_stack.copy_(perm.to(device))
    gd = torch.Generator(device=device).manual_seed(seed + 2)
    # prefill every layer to the start contexts, in chunks of at most 512 tokens per sequence
    done = torch.zeros_like(start)
    while bool((done < start).any()):
        n = torch.clamp(start - done, max=512)
        T = int(n.max())
        cache.begin_step(n)
        for layer in range(L):
            k = torch.randn(B, T, hkv, d, generator=gd, device=device, dtype=torch.float16)
            v = torch.randn(B, T, hkv, d, generator=gd, device=device, dtype=torch.float16)
            if w["kv"] == "int4":  # 1% outliers x8
                k[torch.rand(k.shape, generator=gd, device=device) < 0.01] *= 8
                v[torch.rand(v.shape, generator=gd, device=device) < 0.01] *= 8
            cache.append(layer, k, v)
            del k, v
        done += n
    torch.cuda.synchronize()
    cache.check()
    cache._max_len = max_final
    # per-step inputs (device), distinct per layer
    q = torch.randn(L, B, hq, d, generator=gd, device=device, dtype=torch.float16)
    kn = torch.randn(L, B, 1, hkv, d, generator=gd, device=device, dtype=torch.float16)
    vn = torch.randn(L, B, 1, hkv, d, generator=gd, device=device, dtype=torch.float16)
    out = torch.empty(L, B, hq, d, device=device, dtype=torch.float16)
    return cache, Schedule(ctx, P), max_final, q, kn, vn, out


def launch_floor_ms(w, device, reps=50):
    """Average time of one attention launch, in a graph of the workload's L launches, when every sequence
    holds a single staged token: the fixed per-launch cost (launch, plan records, q load, output write,
    the launch boundary) that every launch of the workload pays on top of its page traffic."""
    L = w["layers"]
    ctx = torch.full((w["batch"],), 2, dtype=torch.int32)
    cache, _, max_ctx, q, _, _, out = build(w, device, seed=7, ctx=ctx)
    cache._decode_plan()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            for layer in range(L):
                cache.attend(layer, q[layer], out=out[layer], max_context=max_ctx)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        g.replay()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    cache.check()
    del g
    return e0.elapsed_time(e1) / (reps * L)


def plan_steps(sched, n, device):
    """Precompute n steps of the schedule: device truncation args + host lengths after each step."""
    plans = []
    for _ in range(n):
        ids, lens, after = sched.next_step()
        if ids is not None:
            ids, lens = ids.to(device), lens.to(device)
        plans.append((ids, lens, after.tolist()))
    return plans


def run_step(cache, q, kn, vn, out, plan, max_context, ev=None):
    """One decode step over all layers; ev: list of (start, end) event pairs around each attention."""
    ids, lens, _ = plan
    if ids is not None:
        cache.truncate(lens, ids)
    cache.begin_step(1)
    for layer in range(cache.num_layers):
        cache.append(layer, kn[layer], vn[layer])
        if ev is not None:
            ev[layer][0].record()
        cache.attend(layer, q[layer], out=out[layer], max_context=max_context)
        if ev is not None:
            ev[layer][1].record()


# --------------------------------------------------------------------------
# CPU path (the reference's CPU implementation, restated in the oracle)
# --------------------------------------------------------------------------

def cpu_sample_gbs(w, seconds=10.0, seed=0):
    """Time the oracle's fp32 numpy CPU path (dequantize pages, then attend --
    the reference's tests/reference.py + torch-CPU path) on whole sequences of
    the same workload until ~``seconds`` pass.  Returns (GB/s, cores, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_cpu

    return oracle_cpu.time_decode_sample(w, seconds=seconds, seed=seed)


# --------------------------------------------------------------------------

def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch(workload):
    """dram bytes per attention launch from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", f"decode_attention_{workload}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def append_sweep(device, kv="int4", batch=64, sizes=(1, 4, 16, 64, 256, 1024, 4096)):
    """KV-append bandwidth of the sharded configuration's shape (TinyLlama
    attention shape, INT4, page 16, 64 sequences) for N new tokens per sequence
    per step: per N, a fresh cache, 2 warm-up steps, then timed steps of one
    allocation launch (begin_step) and one layer's append, CUDA events around
    the steps.  N counts tokens per sequence (N x 64 tokens a step)."""
    from metagross_b200.batched import BatchedPagedKVCache

    w = dict(WORKLOADS["lognormal_int4"], kv=kv)
    P, hkv, d = w["page"], w["hkv"], w["d"]
    rows = []
    for n in sizes:
        steps = max(5, min(200, 20000 // n))
        warm = 2
        total = (steps + warm) * n
        mb = total // P + 2
        cache = BatchedPagedKVCache(1, batch, hkv, d, page_size=P, num_pages=batch * mb, max_blocks=mb, kv_dtype=kv,
                                    staging_dtype=torch.float16, device=device)
        g = torch.Generator(device=device).manual_seed(n)
        k = torch.randn(batch, n, hkv, d, generator=g, device=device, dtype=torch.float16)
        v = torch.randn(batch, n, hkv, d, generator=g, device=device, dtype=torch.float16)
        for _ in range(warm):
            cache.begin_step(n)
            cache.append(0, k, v)
        torch.cuda.synchronize()
        cache.check()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            cache.begin_step(n)
            cache.append(0, k, v)
        e1.record()
        torch.cuda.synchronize()
        cache.check()
        ms = e0.elapsed_time(e1) / steps
        byts = 0.0
        for s_ in range(steps):
            o = (warm + s_) * n
            byts += append_sweep_bytes([o] * batch, [o + n] * batch, w)
        byts /= steps
        rows.append({"n_new": n, "tokens_per_step": n * batch, "ms_per_step": round(ms, 4),
                     "gbs": round(byts / (ms / 1e3) / 1e9, 1), "bytes_per_step": int(byts)})
        del cache, k, v
        torch.cuda.empty_cache()
    return {"metric": "kv append GB/s (N new tokens per sequence per step)", "unit": "GB/s", "kv": kv,
            "config": {"batch": batch, "num_kv_heads": hkv, "head_dim": d, "page": P,
                       "interpretation": "N counts new tokens per sequence; one layer's append + the allocation "
                                         "launch per step, graph-free eager launches"},
            "sweep": rows}


def gather_bench(device, workload="tinyllama_int4", reps=20):
    """The standalone block gather + dequantize (one layer pool of the named
    workload, every sequence, fp16 out): device GB/s over the bytes it must
    move (codes + page scales + block-table entries + staged rows read, fp16
    K/V written), CUDA events over reps launches."""
    from metagross_b200 import _C

    w = dict(WORKLOADS[workload], layers=1)
    cache, _, _, _, _, _, _ = build(w, device, seed=4321)
    lens = cache.seq_lens.cpu()
    cu = torch.zeros(cache.batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    total = int(cu[-1])
    ok = torch.empty(total, cache.num_kv_heads, cache.head_dim, dtype=torch.float16, device=device)
    ov = torch.empty_like(ok)
    cu_d = cu.to(device)
    mc = int(lens.max())

    def run():
        _C.gather_dequant(cache.k_pool[0], cache.v_pool[0], cache.k_scales[0], cache.v_scales[0], cache.staging_k[0],
                          cache.staging_v[0], cache.block_tables, cache.seq_lens, cu_d, mc, ok, ov, cache.status)

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    cache.check()
    ms = e0.elapsed_time(e1) / reps
    bq = 1.0 if w["kv"] == "int8" else 0.5
    P, row = w["page"], w["hkv"] * w["d"]
    byts = 0.0
    for c in lens.tolist():
        n, r = c // P, c % P
        byts += 2 * n * P * row * bq + 8 * n + 4 * n + 2 * r * row * 2 + 2 * c * row * 2
    return {"metric": "gather + dequantize GB/s", "value": round(byts / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "workload": workload, "sequences": cache.batch, "tokens": total, "ms_per_launch": round(ms, 4),
            "bytes_per_launch": int(byts)}


def reference_decode(sequences=2, new_tokens=64, prompt_len=128):
    """The reference's generate_tinyllama_fused on the same architecture
    (baseline/time_reference_decode.py), in a child interpreter whose import
    path holds only the reference install."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    script = os.path.join(ROOT, "baseline", "time_reference_decode.py")
    if not os.path.isdir(os.path.join(ref_dir, "metagross")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    env = dict(os.environ, PYTHONPATH=ref_dir)
    r = subprocess.run([sys.executable, script, "--sequences", str(sequences), "--new-tokens", str(new_tokens),
                        "--prompt-len", str(prompt_len)], cwd=os.path.join(ROOT, "baseline"), env=env,
                       capture_output=True, text=True, timeout=1200)
    for line in r.stdout.splitlines():
        if line.startswith("{"):
            return json.loads(line)
    return {"unavailable": f"reference decode failed (rc {r.returncode}): {r.stderr.strip().splitlines()[-1:]}"}


def decode_model(device, batch=64, prompt_len=128, new_tokens=256, kv="int8"):
    """End-to-end greedy decode of the TinyLlama-1.1B architecture (22 layers,
    hidden 2048, 32 q / 4 kv heads, FFN 5632, vocab 32000, rotary, fp16) with
    seeded random weights on the batched paged cache: prompts of prompt_len
    seeded random token ids, new_tokens tokens per sequence, one CUDA-graph
    decode step per token.  A first pass warms up (cuBLAS, graph upload); the
    cache is reset and the same prompts run again, timed with CUDA events."""
    from metagross_b200.llama import TINYLLAMA_1_1B, LlamaDecoder

    dec = LlamaDecoder(TINYLLAMA_1_1B, batch, prompt_len + new_tokens + 16, kv_dtype=kv, device=device, seed=1234)
    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, TINYLLAMA_1_1B.vocab, (batch, prompt_len), generator=g).to(device)
    dec.prefill(prompt)
    dec.capture()
    dec.decode(8)
    torch.cuda.synchronize()
    dec.cache.reset()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    dec.prefill(prompt)
    ev[1].record()
    toks = dec.decode(new_tokens)
    ev[2].record()
    torch.cuda.synchronize()
    dec.cache.check()
    pre_ms, dec_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    steps = new_tokens - 1  # the first new token comes out of the prefill
    return {"metric": "decode tokens/s", "value": round(batch * steps / (dec_ms / 1e3), 1), "unit": "tokens/s",
            "higher_is_better": True, "dtype": "fp16 model, " + kv + " paged cache", "data": "synthetic",
            "config": {"model": "TinyLlama-1.1B architecture, seeded random weights", "batch": batch,
                       "prompt_len": prompt_len, "new_tokens": new_tokens, "page": 16},
            "decode_ms": round(dec_ms, 2), "ms_per_token_step": round(dec_ms / steps, 4),
            "prefill_ms": round(pre_ms, 2),
            "tokens_per_s_with_prefill": round(batch * new_tokens / ((pre_ms + dec_ms) / 1e3), 1),
            "first_tokens": toks[0, :8].tolist()}


def reference_cuda_leg(cache, w, q, sample_steps=3):
    """The reference's own CUDA path on the same cache, as its wrapper drives it
    (metagross/attention.py:104-134 over csrc/paged_attention.cu:139-255 and
    csrc/quantize.cu:65-120): one ``paged_attention_committed`` call per
    sequence per layer (fp32 q, the sequence's committed pages through its
    block table) and one ``quantize_new_scale`` per committed page for K and
    for V.  The module is the unmodified reference built for sm_100 by its own
    setup.py into baseline/_ref.  Every layer pool is visited in turn (12 x
    50 MB > L2).  The staged tail, which the reference wrapper attends in torch,
    is not timed (so the comparison favours the reference)."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "metagross")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    if w["kv"] != "int8" or w["d"] != 64:
        return {"unavailable": "the reference's committed-page attention is INT8 with head_dim 64 only"}
    # loaded by file path under a private name: this repository's own
    # ``metagross`` package (the drop-in alias) must not shadow it, nor it that
    import glob
    import importlib.util

    so = sorted(glob.glob(os.path.join(ref_dir, "metagross", "_C*.so")))
    if not so:
        return {"unavailable": "reference _C extension missing from baseline/_ref"}
    spec = importlib.util.spec_from_file_location("metagross_reference_build._C", so[0])
    ref_C = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref_C)
    L, B, P = cache.num_layers, cache.batch, cache.page_size
    lens = cache.seq_lens.cpu().tolist()
    tables = [cache.block_tables[b, : lens[b] // P].contiguous() for b in range(B)]
    qf = q.float()
    scale = 1.0 / math.sqrt(w["d"])

    def one_step():
        for layer in range(L):
            for b in range(B):
                ref_C.paged_attention_committed(qf[layer, b], cache.k_pool[layer], cache.v_pool[layer],
                                                cache.k_scales[layer], cache.v_scales[layer], tables[b], scale)

    one_step()  # warm-up
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(sample_steps):
        one_step()
    e1.record()
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3 / sample_steps
    att_ms = e0.elapsed_time(e1) / sample_steps
    # a page commit: quantize_new_scale on a [P, Hkv, D] fp32 page, K and V
    g = torch.Generator(device=q.device).manual_seed(7)
    src = torch.randn(P, w["hkv"], w["d"], generator=g, device=q.device)
    dst = torch.zeros(P, w["hkv"], w["d"], dtype=torch.int8, device=q.device)
    for _ in range(5):
        ref_C.quantize_new_scale(src, dst, 0)
    torch.cuda.synchronize()
    nq = 64
    e0.record()
    for _ in range(nq):
        ref_C.quantize_new_scale(src, dst, 0)
    e1.record()
    torch.cuda.synchronize()
    q_ms = e0.elapsed_time(e1) / nq
    # one decode step commits a page for every sequence every P steps, in every layer, K and V
    step_ms = att_ms + L * B * 2 * q_ms / P
    committed = [(c // P) * P for c in lens]
    att_bytes = L * attention_bytes(committed, w)
    return {"kind": "ref_C_sm100", "module": "metagross._C of the unmodified reference, built for sm_100 by its "
                                              "setup.py into baseline/_ref",
            "ms_per_step": round(step_ms, 4), "attention_ms_per_step": round(att_ms, 4),
            "attention_wall_ms_per_step": round(wall_ms, 4), "quantize_ms_per_call": round(q_ms, 5),
            "attention_calls_per_step": L * B, "attention_gbs": round(att_bytes / (att_ms / 1e3) / 1e9, 1),
            "unit": "GB/s",
            "note": f"{sample_steps} steps x {L} layers x {B} calls (one per sequence, fp32 q, committed pages); "
                    f"quantize_new_scale per committed page (K and V), every {P} steps per sequence; the staged "
                    f"tail (torch in the reference wrapper) not timed"}


def measure(w, name, steps, warmup, world, rank, local, device, e2e=True, equal_counts=True, min_timed_s=1.0):
    """Build the workload on this rank and time it.  Returns a dict of the
    figures (rank-0 aggregates already reduced over ranks)."""
    sharded = bool(w.get("sharded", False))
    gatherer = None
    gather_buf = None
    loads = None
    if sharded:
        # one global batch, split over the ranks by context length (strong scaling)
        from metagross_b200.sharding import ShardGather, lpt_shard, shard_loads

        glob_ctx = contexts_for(w, w["batch"], seed=1234)
        shards = lpt_shard(glob_ctx.numpy(), world, equal_counts=equal_counts)
        loads = shard_loads(glob_ctx.numpy(), shards)
        cache, sched, max_ctx, q, kn, vn, out = build(w, device, seed=1234 + rank,
                                                      ctx=glob_ctx[torch.as_tensor(shards[rank])])
        if world > 1:
            gatherer = ShardGather(shards, rank, (w["hq"], w["d"]), torch.float16, device)
    else:
        # every rank runs the same per-GPU workload on its own sequences (weak scaling)
        cache, sched, max_ctx, q, kn, vn, out = build(w, device, seed=1234 + rank)
        if world > 1:
            gather_buf = torch.empty(world * w["batch"], w["hq"], w["d"], device=device, dtype=torch.float16)
    L, B = w["layers"], cache.batch
    e2e_steps = max(3, steps // 2)
    warm_plans = plan_steps(sched, warmup, device)

    from metagross_b200 import DecodeGraph

    def gather():
        if world > 1:
            import torch.distributed as dist

            if gatherer is not None:
                # every rank's last-layer outputs on every rank: the padded rank-major buffer
                # and the per-rank lengths (the global order is one index_select away)
                gatherer(out[L - 1], reorder=False)
            else:
                dist.all_gather_into_tensor(gather_buf, out[L - 1])

    for pl in warm_plans[:2]:  # eager steps (allocate the workspace and plan buffers)
        run_step(cache, q, kn, vn, out, pl, max_ctx)
        gather()
    graph = DecodeGraph(cache, q, kn, vn, out, n_new=1)

    def step(plan):
        ids, lens, _ = plan
        if ids is not None:
            cache.truncate(lens, ids)
        graph.replay()
        gather()

    t_w0 = time.perf_counter()
    for pl in warm_plans[2:]:
        step(pl)
    torch.cuda.synchronize()
    cache.check()
    # repeats of the K timed steps, so that the clock sampler sees >= min_timed_s of load
    est = (time.perf_counter() - t_w0) / max(1, len(warm_plans) - 2)
    repeats = int(min(200, max(1, math.ceil(min_timed_s / max(steps * est, 1e-6)))))
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([repeats], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        repeats = int(t.item())
    timed_plans = [plan_steps(sched, steps, device) for _ in range(repeats)]
    e2e_plans = plan_steps(sched, e2e_steps, device)

    # bytes of the timed steps (lengths known on the host)
    att_b, app_b = 0.0, 0.0
    n_trunc = 0
    for rp in timed_plans:
        for ids, _, after in rp:
            att_b += L * attention_bytes(after, w)
            app_b += L * append_bytes(after, w)
            n_trunc += ids is not None
    step_bytes = (att_b + app_b) / (steps * repeats)

    clocks = ClockSampler(local)
    clocks.start()
    clocks.mark_start()
    ms_rep = []
    for r in range(repeats):
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for s_ in range(steps):
            step(timed_plans[r][s_])
        t1.record()
        torch.cuda.synchronize()
        ms_rep.append(t0.elapsed_time(t1))
    clocks.mark_stop()
    clk = clocks.stop()
    ms = float(sum(ms_rep)) / repeats  # K steps
    cache.check()

    # ---- the attention kernel alone: a graph of the L attention launches ------------
    # planned as the decode step plans (mg_plan_step, here with no new tokens), so that
    # each launch, settled behind the previous one, copies its first pages before its wait
    cache.begin_step(0, plan=True)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g_att = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g_att, stream=side):
            for layer in range(L):
                cache.attend(layer, q[layer], out=out[layer], max_context=max_ctx)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        g_att.replay()
    att_reps = max(5, min(50, steps // 4))
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a0.record()
    for _ in range(att_reps):
        g_att.replay()
    a1.record()
    torch.cuda.synchronize()
    att_avg_ms = a0.elapsed_time(a1) / (att_reps * L)
    att_lens = timed_plans[-1][-1][2]
    att_bytes_per_launch = attention_bytes(att_lens, w)
    del g_att
    floor_ms = launch_floor_ms(w, device)
    gather_ms = 0.0
    if world > 1:
        import torch.distributed as dist

        # the per-step output gather alone (NCCL over NVLink), reported beside the step
        dist.barrier()
        torch.cuda.synchronize()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(20):
            gather()
        g1.record()
        torch.cuda.synchronize()
        gather_ms = g0.elapsed_time(g1) / 20
        t = torch.tensor([ms, att_avg_ms, gather_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, att_avg_ms, gather_ms = float(t[0]), float(t[1]), float(t[2])

    res = {"ms": ms, "steps": steps, "repeats": repeats, "ms_per_repeat": [round(x, 3) for x in ms_rep],
           "att_avg_ms": att_avg_ms, "att_bytes_per_launch": att_bytes_per_launch, "gather_ms": gather_ms,
           "floor_ms": floor_ms,
           "clk": clk, "n_trunc": n_trunc, "L": L, "sharded": sharded, "loads": loads,
           "att_reps": att_reps, "cache": cache, "q": q}

    # ---- end to end through the public API with host buffers -----------------
    e_bytes = 0.0
    e_ms = None
    if e2e:
        qh = q.cpu().pin_memory()
        knh, vnh = kn.cpu().pin_memory(), vn.cpu().pin_memory()
        outh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        for _, _, after in e2e_plans:
            e_bytes += L * (attention_bytes(after, w) + append_bytes(after, w))
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for s_ in range(e2e_steps):
            q.copy_(qh, non_blocking=True)  # the graph's input buffers, refilled from pinned host memory
            kn.copy_(knh, non_blocking=True)
            vn.copy_(vnh, non_blocking=True)
            step(e2e_plans[s_])
            outh.copy_(out, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        if world > 1:
            import torch.distributed as dist

            t = torch.tensor([e_ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t[0])
        res["e2e_io"] = (int(q.numel() * 2 + kn.numel() * 2 + vn.numel() * 2), int(out.numel() * 2))
    # whole-job totals: every rank's own bytes and sequences, summed
    tot_step_bytes, tot_e_bytes, tot_batch = step_bytes, e_bytes, float(B)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([step_bytes, e_bytes, float(B)], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        tot_step_bytes, tot_e_bytes, tot_batch = float(t[0]), float(t[1]), float(t[2])
    cache.check()
    res.update(tot_step_bytes=tot_step_bytes, tot_e_bytes=tot_e_bytes, tot_batch=tot_batch, e_ms=e_ms,
               e2e_steps=e2e_steps,
               ctx_mean=float(np.mean([np.mean(a) for rp in timed_plans for _, _, a in rp])),
               value=tot_step_bytes / (ms / steps / 1e3) / 1e9)
    graph = None
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="gpt2_int8")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-cuda", action="store_true",
                    help="skip timing the reference's own CUDA ops (baseline/_ref) beside the line")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the 1024-sequence log-normal INT4 strong-scaling figures that ride along with the "
                         "default workload")
    ap.add_argument("--min-timed-s", type=float, default=1.0,
                    help="repeat the K timed steps until the timed region lasts this long (clock sampling)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the workload's layer count (a small case for profiling; the default run uses "
                         "the workload's own depth)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's sequence count (e.g. lognormal_int4 with 128 sequences is one "
                         "rank's share of the 1024 at 8 GPUs)")
    ap.add_argument("--append-sweep", action="store_true",
                    help="instead of the decode benchmark, print the KV-append bandwidth sweep (1..4096 new tokens "
                         "per sequence per step, 64 sequences, INT4) as one JSON line")
    ap.add_argument("--decode-model", action="store_true",
                    help="instead of the decode benchmark, print the end-to-end TinyLlama-architecture greedy decode "
                         "throughput (batch 64, 128-token prompts, 256 new tokens, INT8 cache) as one JSON line")
    ap.add_argument("--new-tokens", type=int, default=256, help="tokens per sequence for --decode-model")
    ap.add_argument("--sweep-sizes", default="1,4,16,64,256,1024,4096",
                    help="new tokens per sequence for --append-sweep (comma-separated)")
    ap.add_argument("--gather", action="store_true",
                    help="instead of the decode benchmark, print the gather + dequantize bandwidth on one layer pool "
                         "of --workload as one JSON line")
    args = ap.parse_args()
    if args.gather:
        print(json.dumps(gather_bench(torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))), args.workload)))
        return
    if args.decode_model:
        line = decode_model(torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))), new_tokens=args.new_tokens)
        if not args.no_reference_cuda:
            ref = reference_decode()
            line["reference_decode"] = ref
            if "value" in ref:
                line["speedup_vs_reference_decode"] = round(line["value"] / ref["value"], 1)
        print(json.dumps(line))
        return
    if args.append_sweep:
        print(json.dumps(append_sweep(torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))),
                                      sizes=tuple(int(x) for x in args.sweep_sizes.split(",")))))
        return
    w = dict(WORKLOADS[args.workload])
    if args.layers is not None:
        if args.layers < 1:
            raise SystemExit("--layers must be >= 1")
        w["layers"] = args.layers
    if args.batch is not None:
        if args.batch < 1:
            raise SystemExit("--batch must be >= 1")
        w["batch"] = args.batch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "paged decode attn HBM GB/s"

    if args.impl == "reference":
        if rank != 0:
            return
        gbs, cores, sample = cpu_sample_gbs(w, seconds=max(1.0, min(args.cpu_seconds, 30.0)))
        line = {"impl": "reference", "metric": metric, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": args.workload, "desc": w["desc"]},
                "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    m = measure(w, args.workload, args.steps, args.warmup, world, rank, local, device,
                min_timed_s=args.min_timed_s)
    ref_cuda = None
    if world == 1 and rank == 0 and not args.no_reference_cuda and args.workload == "gpt2_int8":
        ref_cuda = reference_cuda_leg(m["cache"], w, m["q"])
    m["cache"] = m["q"] = None
    torch.cuda.empty_cache()

    # the 1024-sequence log-normal INT4 configuration, split over the ranks by
    # total tokens (strong scaling), beside the default workload at every N
    sharded_fig = None
    if not args.no_sharded and args.workload == "gpt2_int8" and args.layers is None:
        ws = dict(WORKLOADS["lognormal_int4"])
        c5 = measure(ws, "lognormal_int4", args.steps, args.warmup, world, rank, local, device, e2e=False,
                     equal_counts=False, min_timed_s=0.25)
        lds = c5["loads"]
        sharded_fig = {
            "workload": "lognormal_int4", "desc": ws["desc"], "scaling": "strong",
            "value": round(c5["value"], 1), "unit": "GB/s", "ms_per_step": c5["ms"] / c5["steps"],
            "steps": c5["steps"], "timed_repeats": c5["repeats"],
            "attention_avg_launch_ms": c5["att_avg_ms"],
            "gather_ms_per_step": round(c5["gather_ms"], 4) if world > 1 else None,
            "rank_token_loads": lds, "load_max_over_mean": round(max(lds) / (sum(lds) / len(lds)), 4),
            "split": "LPT on context length (token-balanced, unequal sequence counts); padded all-gather of the "
                     "last layer's outputs plus per-rank lengths",
            "clocks": c5["clk"]}
        c5["cache"] = c5["q"] = None
        torch.cuda.empty_cache()

    if rank == 0:
        peak, peak_kind = peaks()
        L = m["L"]
        achieved = m["att_bytes_per_launch"] / (m["att_avg_ms"] / 1e3) / 1e9
        seq_steps = m["tot_batch"] * args.steps / (m["ms"] / 1e3)
        # which attention kernel ran: every workload here has 16-token pages, page scales, fp16 staging and
        # head_dim 64, so the pool's code width decides (the rule of tma_mode in csrc/mg_attention.cu)
        force = os.environ.get("METAGROSS_B200_ATTENTION", "")
        if force == "registers":
            kernel = "paged_decode_kernel"
        elif w["kv"] == "int8" or force == "bulk":
            kernel = "paged_decode_tma_kernel"
        else:
            kernel = "paged_decode_tma_kernel (self-copying mode)"
        line = {
            "metric": metric, "value": round(m["value"], 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": m["ms"] / args.steps, "higher_is_better": True,
            "scaling": "strong" if m["sharded"] else "weak",
            "vs_baseline": None, "dtype": w["kv"] if w["kv"] == "int8" else "int4", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["desc"], "global_batch": int(m["tot_batch"]),
                       "context_mean": round(m["ctx_mean"], 1), "truncations_timed": m["n_trunc"],
                       "layers": L, "parallelism": f"sequence-sharded dp{world}",
                       "l2": "working set per step > 126 MB L2 (one pool per layer); no flush"},
            "timed_repeats": m["repeats"], "ms_per_repeat": m["ms_per_repeat"],
            "sequence_steps_per_s": round(seq_steps, 1),
            "bytes_per_step": m["tot_step_bytes"],
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic_per_launch(args.workload),
                         "kernel": kernel, "algorithmic_bytes_per_launch": m["att_bytes_per_launch"],
                         "avg_launch_ms": m["att_avg_ms"],
                         "launch_floor_ms": round(m["floor_ms"], 5),
                         "floor_note": "the same graph of attention launches with one staged token per sequence: "
                                       "the fixed cost each launch pays on top of its page traffic",
                         "timing": f"graph of the {L} attention launches (one per layer pool), CUDA events, "
                                   f"{m['att_reps']} replays"},
            "e2e": {"value": round(m["tot_e_bytes"] / (m["e_ms"] / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": m["e2e_io"][0], "d2h_bytes_per_step": m["e2e_io"][1],
                    "ms_per_step": m["e_ms"] / m["e2e_steps"]},
            "gather_ms_per_step": round(m["gather_ms"], 4) if world > 1 else None,
            "gpu_launches": m["repeats"] * args.steps * (2 + 2 * L) + m["n_trunc"],
            "clocks": m["clk"],
        }
        if ref_cuda is not None:
            if "ms_per_step" in ref_cuda:
                ref_cuda["value"] = round(m["tot_step_bytes"] / (ref_cuda["ms_per_step"] / 1e3) / 1e9, 1)
                ref_cuda["step_speedup_of_this_line"] = round(ref_cuda["ms_per_step"] / (m["ms"] / args.steps), 1)
            line["reference_cuda"] = ref_cuda
        if sharded_fig is not None:
            line["sharded_lognormal_int4"] = sharded_fig
        if world == 1 and not args.no_cpu_baseline:
            gbs, cores, sample = cpu_sample_gbs(w, seconds=args.cpu_seconds)
            line["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle_cpu

            c1, c1_threads, c1_desc, c1_ms = oracle_cpu.time_cpu_reference_config(
                seconds=max(2.0, min(args.cpu_seconds, 10.0)))
            line["cpu_baseline_reference_config"] = {"value": round(c1, 4), "unit": "GB/s", "ms_per_step": c1_ms,
                                                     "cores": c1_threads, "kind": "port", "sample": c1_desc}
        print(json.dumps(line), flush=True)

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
