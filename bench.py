#!/usr/bin/env python
"""Decode throughput of the B200 engine on the Qwen3-0.6B architecture.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload batched-int8|bs1-f32|bs1-int8] [--prompt P]
                    [--no-extras] [--no-cpu]

Headline workload (default, every N): batched independent-sequence INT8
decode -- 64 sequences per GPU, each with a 2048-token uniform-random prompt,
then greedy decode; weights replicated per GPU, sequences sharded, no
collective on the token path (weak scaling).  One step = one decode token for
all 64 sequences of every GPU.  value = tokens/s over all GPUs, timed with
CUDA events on the engine's stream over exactly K graph-replayed steps after
W warm-up steps, max over ranks.

At N=1 rank 0 also reports, in the same JSON line:
  bs1_f32  -- batch-1 f32 decode, 32-token prompt + 128 greedy tokens
  bs1_int8 -- batch-1 INT8 decode, 512-token prompt + 512 greedy tokens
and the CPU baseline: the reference engine itself (oracle/_ref, compiled from
its own sources) timed on this host's cores on a bounded sample.

--impl reference times the reference's CPU implementation (Model::step of
oracle/_ref) on the same workload and prints the same JSON line with
"impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "verbum.cpp_b200"), str(ROOT / "oracle")]

METRIC = "Qwen3-0.6B decode tok/s (bs1 f32/int8; batched 1-8 GPU) + % HBM roofline"
WEIGHT_SEED = 1234
FALLBACK_HBM_GBS = 6650.0
KV_BYTES_PER_POS = 28 * 2 * 8 * 128 * 4  # 229,376 B: K and V rows of all layers


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel, units):
    """DRAM bytes (read + write) per launch from an ncu capture of `kernel`
    (profiles/ncu_traffic.json), scaled to `units` by proportion: the kernel
    streams each sequence-position once, so its traffic grows linearly."""
    try:
        d = json.loads((ROOT / "profiles" / "ncu_traffic.json").read_text())[kernel]
        return int(d["dram_bytes_per_launch"] * units / d["units_per_launch"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                if int(f[0]) not in self.gpus:
                    continue
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "power_w_max": max(power), "samples": len(sm), "reasons": sorted(reasons)}


def write_model(tmpdir, cfg, weights):
    import vbsynth
    return vbsynth.write_model_dir(Path(tmpdir) / "qwen3-0.6b-synth", cfg, weights)


# ---------------------------------------------------------------------------
# reference (CPU) timing -- oracle/_ref is the reference engine itself
# ---------------------------------------------------------------------------

def _ref_worker(args):
    model_dir, mode, ctx, warm, steps, first_token = args
    import oracle
    m = oracle.RefModel(model_dir)
    if mode == "int8":
        m.quantize()
    m.reset_cache(ctx + warm + steps + 8)
    m.set_cache_len(ctx)
    if warm:
        m.greedy_steps(first_token, warm)
    _, secs = m.greedy_steps(first_token, steps)
    m.close()
    return [float(s) for s in secs]


def ref_time(model_dir, mode, ctx, warm, steps, procs):
    """Times Model::step of the reference at context length ctx on `procs`
    single-threaded processes (the engine is single-threaded), each decoding
    its own sequence.  Returns (aggregate tok/s, per-step seconds)."""
    jobs = [(str(model_dir), mode, ctx, warm, steps, 1000 + i) for i in range(procs)]
    with mp.get_context("spawn").Pool(procs) as pool:
        res = pool.map(_ref_worker, jobs)
    per_proc_rate = [len(r) / sum(r) for r in res]
    return sum(per_proc_rate), [s for r in res for s in r]


def ref_procs(max_procs=16, gb_per_proc=5.0):
    n = os.cpu_count() or 1
    try:
        import psutil
        avail = psutil.virtual_memory().available / 1e9
        n = min(n, max(1, int(avail // gb_per_proc)))
    except Exception:
        pass
    return max(1, min(n, max_procs))


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# GPU workloads
# ---------------------------------------------------------------------------

def step_kv_bytes(n_ctx):
    """KV traffic of one decode step at context n_ctx (reads n_ctx rows incl.
    the new one, writes 1)."""
    return KV_BYTES_PER_POS * (n_ctx + 1)


def run_prefill(args, weights, cfg, dev=0):
    """The batched prefill alone (B sequences x P prompt positions, INT8 model):
    device time with CUDA events on the engine stream, prompt tokens/s."""
    import numpy as np
    import torch

    import vb200
    import vbsynth

    B, P = args.batch, args.prompt
    torch.cuda.set_device(dev)
    eng = vb200.Engine(cfg, device=dev).load(weights)
    eng.quantize()
    bt = vb200.Batch(eng, B, P + 8)
    prompts = np.stack([vbsynth.prompt_ids(P, 77 + b, cfg["vocab_size"]) for b in range(B)])
    bt.prefill(prompts[:, :64].T.copy())  # builds the tensor-core weight copies
    bt.reset()
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0.record(stream)
    nx = bt.prefill(prompts.T.copy())
    ev1.record(stream)
    ev1.synchronize()
    wall = time.perf_counter() - t0
    sec = ev0.elapsed_time(ev1) / 1e3
    out = {"batch": B, "prompt": P, "seconds": round(sec, 4), "wall_s": round(wall, 4),
           "prompt_tok_s": round(B * P / sec, 1), "first_next": [int(x) for x in nx[:4]]}
    bt.close()
    eng.close()
    return out


def run_batched(args, grp, weights, cfg):
    import numpy as np
    import torch

    import vb200
    import vbdist
    import vbsynth

    B = args.batch
    P = args.prompt
    K, W = args.steps, args.warmup
    dev = grp.local_rank
    torch.cuda.set_device(dev)
    eng = vb200.Engine(cfg, device=dev).load(weights)
    eng.quantize()
    bt = vb200.Batch(eng, B, P + W + 2 * K + 8)
    gidx = list(vbdist.shard(B * grp.world, grp.rank, grp.world))
    prompts = np.stack([vbsynth.prompt_ids(P, vbdist.sequence_seed(g), cfg["vocab_size"])
                        for g in gidx])
    # the first prefill also converts the weights for the tensor cores, sizes
    # the prefill buffers and builds the decode step's graph; the prompt is
    # prefilled again after a reset for the steady-state time
    t0 = time.perf_counter()
    nx = bt.prefill(prompts.T.copy())
    prefill_first_s = time.perf_counter() - t0
    bt.reset()
    t0 = time.perf_counter()
    nx = bt.prefill(prompts.T.copy())
    prefill_s = time.perf_counter() - t0
    if W:
        nx = bt.decode(nx, W)
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(list(range(grp.world)) if grp.world > 1 else [dev]).start() \
        if grp.rank == 0 else None
    nx0, len0 = nx.copy(), bt.cache_len()
    # R repeats of the same K timed steps (the caches are rolled back to where
    # the first repeat started, so every repeat decodes the same positions);
    # the line reports the median repeat, max over ranks within each repeat
    ms_reps = []
    for _ in range(args.repeats):
        bt.truncate(len0)
        grp.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        nx = bt.decode(nx0, K)
        ev1.record(stream)
        ev1.synchronize()
        torch.cuda.synchronize()
        grp.barrier()
        ms_reps.append(grp.reduce_max(ev0.elapsed_time(ev1)))
    nx_dev = nx.copy()
    # end to end through the C ABI with host buffers (tokens in, next tokens
    # out, one call per step) over the same K steps at the same positions
    e2e_reps = []
    for _ in range(args.repeats):
        bt.truncate(len0)
        nx = nx0
        grp.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(K):
            _, nx = bt.step(nx, want_logits=False, want_next=True)
        e2e_reps.append(grp.reduce_max(time.perf_counter() - t0))
        if not np.array_equal(nx, nx_dev):
            raise SystemExit("batched decode: per-step API and device loop disagree")
    grp.barrier()
    clocks = clk.stop() if clk else None
    ms = statistics.median(ms_reps)
    e2e_s = statistics.median(e2e_reps)
    checksum = grp.gather_ints([int(x) for x in nx[:4]])
    n_mid = P + W + K // 2
    res = {
        "ms": ms, "e2e_s": e2e_s, "prefill_s": grp.reduce_max(prefill_s),
        "prefill_first_s": grp.reduce_max(prefill_first_s),
        "ms_repeats": [round(x, 3) for x in ms_reps], "e2e_s_repeats": [round(x, 4) for x in e2e_reps],
        "graph_nodes": bt.graph_nodes(), "n_mid": n_mid, "clocks": clocks,
        "checksum": checksum, "weight_bytes": eng.weight_bytes(),
    }
    # dominant kernel: split-K attention over the 64 caches, timed standalone on
    # this workload's shape at the mid context (28 launches = one step's worth)
    res["attn"] = time_attention(B, n_mid, dev, launches=28)
    bt.close()
    eng.close()
    return res


def time_attention(B, n, dev, launches=28, H=16, KVH=8, D=128):
    import torch

    import vb200
    g = torch.Generator(device=f"cuda:{dev}").manual_seed(5)
    q = torch.randn(B, H, D, device=f"cuda:{dev}", generator=g)
    # [B, KVH, n, D]: the engine's cache layout
    k = torch.randn(B, KVH, n, D, device=f"cuda:{dev}", generator=g)
    v = torch.randn(B, KVH, n, D, device=f"cuda:{dev}", generator=g)
    lens = torch.full((B,), n, dtype=torch.int32, device=f"cuda:{dev}")
    out = torch.empty(B, H, D, device=f"cuda:{dev}")
    ws = torch.empty(vb200.attn_workspace_bytes(B, H, n) // 4 + 1, device=f"cuda:{dev}")
    s = torch.cuda.current_stream(dev)
    args = (q, k, v, out, lens, B, H, KVH, D, n, KVH * n * D, D, n * D, ws)
    for _ in range(3):
        vb200.attn_decode_batched(*args, stream=s.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(launches):
        vb200.attn_decode_batched(*args, stream=s.cuda_stream)
    e1.record(s)
    e1.synchronize()
    per = e0.elapsed_time(e1) / launches / 1e3
    bytes_ = B * n * KVH * D * 4 * 2
    del k, v
    torch.cuda.empty_cache()
    return {"kernel": "attn_split_kernel<2> + attn_merge_kernel", "sec_per_launch": per,
            "bytes_per_launch": bytes_, "B": B, "n": n}


GEMV_SHAPES = [("q", 1024, 2048), ("k", 1024, 1024), ("v", 1024, 1024), ("o", 2048, 1024),
               ("gate", 1024, 3072), ("up", 1024, 3072), ("down", 3072, 1024),
               ("lm_head", 1024, 151936)]


def _graph_time(fn, launches, dev):
    """Captures `launches` calls of fn(i) in one CUDA graph and times its replay
    with CUDA events (back-to-back launches, no host overhead between them)."""
    import torch
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    e1.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / (reps * launches)
    del g
    return sec


def gemv_microbench(dev=0, shapes=None, dtypes=("f32", "int8"), min_bytes=2 * 126 * 2**20):
    """Config 2: each GEMV shape, f32 and INT8, rotating through enough weight
    copies that the weights come from HBM (>= 2x L2 per rotation)."""
    import torch

    import vb200
    out = {}
    for name, K, N in (shapes or GEMV_SHAPES):
        for dt in dtypes:
            wbytes = N * K * (4 if dt == "f32" else 1) + (0 if dt == "f32" else 4 * N)
            copies = max(1, -(-min_bytes // wbytes))
            x = torch.randn(1, K, device=f"cuda:{dev}")
            y = torch.empty(1, N, device=f"cuda:{dev}")
            if dt == "f32":
                Ws = [torch.randn(N, K, device=f"cuda:{dev}") * 0.02 for _ in range(copies)]
                fn = lambda i: vb200.matmul_nt_f32(x, Ws[i % copies], y,
                                                   stream=torch.cuda.current_stream().cuda_stream)
            else:
                Ws = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=f"cuda:{dev}")
                      for _ in range(copies)]
                sc = [torch.rand(N, device=f"cuda:{dev}") * 1e-3 for _ in range(copies)]
                fn = lambda i: vb200.matmul_nt_q8(x, Ws[i % copies], sc[i % copies], y,
                                                  stream=torch.cuda.current_stream().cuda_stream)
            launches = max(copies * 2, 20)
            sec = _graph_time(fn, launches, dev)
            alg = wbytes + 4 * K + 4 * N
            out[f"{name}_{dt}"] = {"K": K, "N": N, "us": round(sec * 1e6, 2),
                                   "gbs": round(alg / sec / 1e9, 1)}
            del Ws
            torch.cuda.empty_cache()
    return out


def attn_microbench(dev=0, ns=(512, 2048, 8192, 32768), Bs=(1, 32), H=16, KVH=8, D=128):
    """Config 4: isolated GQA decode attention, K/V [B, n, 8, 128] f32 ~ N(0,1),
    RoPE pre-applied; GB/s on KV reads (each KV head read once)."""
    import torch

    import vb200
    out = {}
    for B in Bs:
        for n in ns:
            g = torch.Generator(device=f"cuda:{dev}").manual_seed(n + B)
            q = torch.randn(B, H, D, device=f"cuda:{dev}", generator=g)
            k = torch.randn(B, n, KVH, D, device=f"cuda:{dev}", generator=g)
            v = torch.randn(B, n, KVH, D, device=f"cuda:{dev}", generator=g)
            lens = torch.full((B,), n, dtype=torch.int32, device=f"cuda:{dev}")
            o = torch.empty(B, H, D, device=f"cuda:{dev}")
            ws = torch.empty(vb200.attn_workspace_bytes(B, H, n) // 4 + 1, device=f"cuda:{dev}")
            kv_bytes = B * n * KVH * D * 4 * 2
            launches = max(4, min(64, int(4e9 // kv_bytes)))

            def fn(i):
                vb200.attn_decode_batched(q, k, v, o, lens, B, H, KVH, D, n, n * KVH * D, KVH * D,
                                          D, ws, stream=torch.cuda.current_stream().cuda_stream)
            sec = _graph_time(fn, launches, dev)
            out[f"B{B}_n{n}"] = {"us": round(sec * 1e6, 2), "gbs": round(kv_bytes / sec / 1e9, 1),
                                 "kv_bytes": kv_bytes}
            del k, v
            torch.cuda.empty_cache()
    return out


STEPS2 = ("A.poll", "A.norm", "A.qkv", "A.gather", "A.attn", "A.merge", "A.oproj",
          "B.poll", "B.norm", "B.gateup", "B.down", "B.reduce")


def trace_breakdown2(tr, layers=28, stride=2048):
    """Two-barrier step: median (over layers and the CTAs of the kv clusters)
    duration of each of the 12 marked steps of a layer, and the median layer
    time, in us."""
    import numpy as np
    G = len(tr) // stride
    if G == 0:
        return None
    t = np.asarray(tr, dtype=np.int64).reshape(G, stride).astype(np.float64)
    m = t[:, 1:1 + 12 * layers].reshape(G, layers, 12)
    full = (m != 0).all(axis=(1, 2)) & (t[:, 0] != 0)
    if not full.any():
        return None
    t, m = t[full], m[full]
    prev = np.concatenate([t[:, :1, None], m[:, :-1, 11:12]], axis=1)  # [G, L, 1]
    d = np.diff(np.concatenate([prev, m], axis=2), axis=2)  # [G, L, 12]
    out = {name: round(float(np.median(d[:, :, i])) / 1e3, 2) for i, name in enumerate(STEPS2)}
    out["layer_us"] = round(float(np.median(m[:, 1:, 11] - m[:, :-1, 11])) / 1e3, 2)
    out["total_us"] = round(float(m[:, -1, 11].max() - t[:, 0].min()) / 1e3, 1)
    out["ctas"] = int(G)
    # cycle profile of consumer thread 0 (words 400 + 16*l)
    pr = t[:, 400:400 + 40 * layers].reshape(-1, layers, 40)
    dc = pr[:, 1:, 14] - pr[:, :-1, 14]
    dn = pr[:, 1:, 15] - pr[:, :-1, 15]
    ok = dn > 0
    if ok.any():
        ghz = float(np.median(dc[ok] / dn[ok]))
        out["sm_ghz"] = round(ghz, 3)
        names = ["qkv.wait", "qkv.all", "o.wait", "o.all", "gu.wait", "gu.all", "d.wait", "d.all",
                 "x.gather", "x.merge", "x.reduce", "attn.wait", "-", "attn", "-", "-",
                 "qkv.first", "qkv.dot", "qkv.epi", "o.first", "o.dot", "o.epi", "gu.first", "gu.dot", "gu.epi"]
        out["cycles_us"] = {n: round(float(np.median(pr[:, :, i])) / ghz / 1e3, 3)
                            for i, n in enumerate(names) if n != "-"}
        busy = pr[:, :, 12] > 0  # CTAs whose warp 0 had attention chunks
        if busy.any():
            out["cycles_us"]["attn.busy"] = round(float(np.median(pr[:, :, 13][busy])) / ghz / 1e3, 3)
            out["cycles_us"]["attn.busy_wait"] = round(float(np.median(pr[:, :, 11][busy])) / ghz / 1e3, 3)
            out["cycles_us"]["attn.chunks"] = round(float(np.median(pr[:, :, 12][busy])), 1)
    return out


def profile_batched(batch, prompt_len, n_steps, weights, cfg, dev=0):
    """For ncu --profile-from-start off: n_steps decode steps of the batched
    INT8 workload bracketed by cudaProfilerStart/Stop after the prompts and a
    warm-up, so a launch list holds exactly those steps' kernels."""
    import numpy as np
    import torch

    import vb200
    import vbdist
    import vbsynth
    eng = vb200.Engine(cfg, device=dev).load(weights)
    eng.quantize()
    bt = vb200.Batch(eng, batch, prompt_len + n_steps + 16)
    prompts = np.stack([vbsynth.prompt_ids(prompt_len, vbdist.sequence_seed(b), cfg["vocab_size"])
                        for b in range(batch)])
    nx = bt.prefill(prompts.T.copy())
    nx = bt.decode(nx, 4)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    bt.decode(nx, n_steps)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    out = {"batch": batch, "prompt": prompt_len, "steps": n_steps, "graph_nodes": bt.graph_nodes()}
    bt.close()
    eng.close()
    return out


def profile_bs1(mode, prompt_len, n_tokens, weights, cfg, dev=0, path=-1):
    """For ncu --profile-from-start off: n_tokens greedy decode steps bracketed
    by cudaProfilerStart/Stop after the prompt and a warm-up, so a launch list
    holds exactly those steps' kernels."""
    import numpy as np
    import torch

    import vb200
    import vbsynth
    e = vb200.Engine(cfg, device=dev).load(weights)
    if mode == "int8":
        e.quantize()
    e.set_path(path)
    prompt = vbsynth.prompt_ids(prompt_len, 77 + prompt_len, cfg["vocab_size"])
    e.reset_cache(prompt_len + n_tokens + 16)
    lg = e.prefill(prompt, want_logits=True)
    tok = int(e.decode(int(np.argmax(lg)), 8)[-1])
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    e.decode(tok, n_tokens)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    out = {"mode": mode, "path": e.path(), "graph_nodes": e.graph_nodes(), "tokens": n_tokens}
    e.close()
    return out


def run_bs1(mode, prompt_len, n_new, weights, cfg, dev=0, warm=8, path=-1, trace=False, lm8=False):
    import numpy as np
    import torch

    import vb200
    import vbsynth
    e = vb200.Engine(cfg, device=dev).load(weights)
    if mode == "int8":
        e.quantize()
    if lm8:
        e.quantize_lm_head()
    e.set_path(path)
    prompt = vbsynth.prompt_ids(prompt_len, 77 + prompt_len, cfg["vocab_size"])
    max_seq = prompt_len + n_new + 8
    # warm-up pass
    e.reset_cache(max_seq)
    lg = e.prefill(prompt, want_logits=True)
    e.decode(int(np.argmax(lg)), warm)
    # timed pass: n_new greedy tokens, device-side feedback
    e.reset_cache(max_seq)
    lg = e.prefill(prompt, want_logits=True)
    first = int(np.argmax(lg))
    stream = torch.cuda.ExternalStream(e.stream(), device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    toks = e.decode(first, n_new)
    ev1.record(stream)
    ev1.synchronize()
    sec = ev0.elapsed_time(ev1) / 1e3
    # the same decode with the reference's default sampler (T 0.8, top-k 40,
    # top-p 0.95) on the device
    smp = vb200.Sampler(0.8, 40, 0.95, 1234)
    e.reset_cache(max_seq)
    e.prefill(prompt)
    e.decode_sampled(smp, first, warm)  # sizes the sampler's buffers
    e.reset_cache(max_seq)
    e.prefill(prompt)
    torch.cuda.synchronize()
    ev0.record(stream)
    e.decode_sampled(smp, first, n_new)
    ev1.record(stream)
    ev1.synchronize()
    sec_sampled = ev0.elapsed_time(ev1) / 1e3
    smp.close()
    # end to end, reference semantics: step(token) -> logits in host memory
    e.reset_cache(max_seq)
    e.prefill(prompt)
    tok = first
    t0 = time.perf_counter()
    lat = []
    for _ in range(n_new):
        t1 = time.perf_counter()
        lg = e.step(tok)
        lat.append(time.perf_counter() - t1)
        tok = int(np.argmax(lg))
    e2e = time.perf_counter() - t0
    wb = e.weight_bytes()
    if lm8:  # the lm_head read as int8 rows + f32 scales instead of the f32 table
        V, H = cfg["vocab_size"], cfg["hidden_size"]
        wb = wb - 4 * V * H + V * H + 4 * V
    nodes = e.graph_nodes()
    engine_path = e.path()
    tb = None
    if trace and e.path() == 2:
        e.set_trace(True)
        e.reset_cache(max_seq)
        e.prefill(prompt)
        e.decode(tok, 4)
        raw = e.read_trace()
        if os.environ.get("VB_TRACE_DUMP"):
            import numpy as np
            np.save(os.environ["VB_TRACE_DUMP"] + f"_{mode}.npy", raw)
        tb = trace_breakdown2(raw, cfg["num_hidden_layers"])
    e.close()
    mean_ctx = prompt_len + (n_new - 1) / 2.0
    bytes_tok = wb + step_kv_bytes(mean_ctx)
    lat.sort()
    return {"tok_s": n_new / sec, "ms_per_token": 1e3 * sec / n_new, "bytes_per_token": bytes_tok,
            "achieved_gbs": bytes_tok * n_new / sec / 1e9, "e2e_tok_s": n_new / e2e,
            "e2e_p50_ms": 1e3 * lat[len(lat) // 2], "e2e_p99_ms": 1e3 * lat[min(len(lat) - 1, int(0.99 * len(lat)))],
            "sampled_tok_s": round(n_new / sec_sampled, 2),
            "graph_nodes": nodes, "weight_bytes": wb, "prompt": prompt_len, "decode_tokens": n_new,
            "engine_path": engine_path,
            "path": "clustered persistent step" if nodes == 1 else "per-op CUDA graph",
            "first_tokens": [int(t) for t in toks[:4]], **({"trace": tb} if tb else {})}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def workload_config(args, n_gpus):
    """The `config` object of the JSON line (identical for both arms)."""
    B, K = args.batch, args.steps
    return {
        "workload": f"batched-int8: {B} independent sequences per GPU, {args.prompt}-token "
                    f"prompts, greedy decode steps {args.warmup}+{K} (warm-up+timed)",
        "model": "Qwen3-0.6B architecture (28 layers, hidden 1024, 16/8 heads, D 128, "
                 "ffn 3072, vocab 151936, tied)",
        "global_batch": B * n_gpus, "seq_len": args.prompt + args.warmup + K,
        "parallelism": f"replicas x{n_gpus}: sequences sharded, weights replicated, no collective",
        "l2": "inputs larger than L2 (>=1.06 GB of weights and ~32 GB of KV per step)",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--repeats", type=int, default=3,
                    help="timed repeats of the K steps (median reported)")
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["batched-int8"], default="batched-int8")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--no-extras", action="store_true", help="skip the bs1 lines")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--only", choices=["gemv", "attn", "bs1", "prefill", "batched"],
                    help="one workload (for profiling)")
    ap.add_argument("--mode", choices=["f32", "int8"], default="int8", help="--only bs1: weights")
    ap.add_argument("--path", type=int, default=-1,
                    help="--only bs1: 1 per-op graph, 2 clustered step, -1 the engine's automatic choice")
    ap.add_argument("--trace", action="store_true",
                    help="--only bs1: per-phase trace of the clustered step (needs a VB_STEP_TRACE=1 build)")
    ap.add_argument("--profile", type=int, default=0,
                    help="--only bs1 / batched: decode this many tokens (steps) inside "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off) instead of the timed run")
    ap.add_argument("--ctx", type=int, default=2048, help="--only attn: context length")
    ap.add_argument("--shape", default=None, help="--only gemv: one of q,k,v,o,gate,up,down,lm_head")
    args = ap.parse_args()
    if args.warmup < 0 or args.steps <= 0:
        raise SystemExit("--steps must be > 0")

    import vbdist
    rank, world, local_rank = vbdist.env_rank()
    if args.impl == "reference":
        return main_reference(args, rank, world)
    if args.only == "gemv":
        shapes = [s for s in GEMV_SHAPES if args.shape in (None, s[0])]
        print(json.dumps({"gemv": gemv_microbench(local_rank, shapes)}), flush=True)
        return 0
    if args.only == "bs1":
        import vbsynth
        cfg = vbsynth.qwen3_config()
        w = vbsynth.make_weights(cfg, seed=WEIGHT_SEED)
        P, G = (32, 128) if args.mode == "f32" else (512, 512)
        if args.profile:
            print(json.dumps({"bs1_profile": profile_bs1(args.mode, P + G // 2, args.profile, w, cfg,
                                                         dev=local_rank, path=args.path)}), flush=True)
            return 0
        r = run_bs1(args.mode, P, min(G, args.steps), w, cfg, dev=local_rank, path=args.path,
                    trace=args.trace)
        print(json.dumps({"bs1": r}), flush=True)
        return 0
    if args.only == "batched":
        import vbsynth
        cfg = vbsynth.qwen3_config()
        w = vbsynth.make_weights(cfg, seed=WEIGHT_SEED)
        print(json.dumps({"batched_profile": profile_batched(args.batch, args.prompt, max(1, args.profile), w, cfg,
                                                             dev=local_rank)}), flush=True)
        return 0
    if args.only == "prefill":
        import vbsynth
        cfg = vbsynth.qwen3_config()
        w = vbsynth.make_weights(cfg, seed=WEIGHT_SEED)
        print(json.dumps({"prefill": run_prefill(args, w, cfg, dev=local_rank)}), flush=True)
        return 0
    if args.only == "attn":
        print(json.dumps({"attn": attn_microbench(local_rank, ns=(args.ctx,), Bs=(args.batch,))}),
              flush=True)
        return 0

    # CPU-baseline processes are spawned before any GPU work
    import vbsynth
    cfg = vbsynth.qwen3_config()
    weights = vbsynth.make_weights(cfg, seed=WEIGHT_SEED)
    grp = vbdist.Group()
    peak, peak_kind = hbm_peak()

    res = run_batched(args, grp, weights, cfg)
    B, K, N = args.batch, args.steps, grp.world
    sec = res["ms"] / 1e3
    value = N * B * K / sec
    attn = res["attn"]
    a_gbs = attn["bytes_per_launch"] / attn["sec_per_launch"] / 1e9
    step_bytes = res["weight_bytes"] + B * step_kv_bytes(res["n_mid"])
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": N,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(res["ms"] / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "weights": "int8 (per-row absmax) projections, f32 embedding/lm_head",
        "data": "synthetic: seeded N(0,0.02) random-init weights, uniform random prompt ids",
        "config": workload_config(args, N),
        "step_roofline_frac": round(step_bytes / (sec / K) / 1e9 / peak, 4),
        "step_bytes": step_bytes,
        "roofline": {
            "bound": "hbm", "kernel": attn["kernel"],
            "achieved": round(a_gbs, 1), "peak": peak, "unit": "GB/s",
            "frac": round(a_gbs / peak, 4), "peak_kind": peak_kind,
            "traffic": ncu_traffic("attn_split_kernel", attn["B"] * attn["n"]),
            "algorithmic_bytes_per_launch": attn["bytes_per_launch"],
            "launch_shape": f"B={attn['B']} n={attn['n']} KVH=8 D=128 f32",
        },
        "clocks": res["clocks"],
        "e2e": {"value": round(N * B * K / res["e2e_s"], 2), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B * N, "d2h_bytes_per_step": 4 * B * N,
                "api": "vb_batch_step (host token ids in, host greedy ids out, per step)"},
        "gpu_launches": res["graph_nodes"] * K,
        "repeats": {"n": args.repeats, "reported": "median",
                    "ms_per_step": [round(x / K, 4) for x in res["ms_repeats"]],
                    "e2e_tok_s": [round(N * B * K / x, 1) for x in res["e2e_s_repeats"]]},
        "prefill_s": round(res["prefill_s"], 3),
        "prefill_first_s": round(res["prefill_first_s"], 3),
        "prefill_tok_s": round(N * B * args.prompt / res["prefill_s"], 1),
    }
    if grp.rank == 0 and N == 1 and not args.no_extras:
        names = {1: "per-op CUDA graph", 2: "clustered step, tagged exchange"}
        for mode, P, G in (("f32", 32, 128), ("int8", 512, 512)):
            # the engine's automatic path (what a Model::step caller gets) is the
            # reported line; the other path is timed on the same inputs beside it
            r_auto = run_bs1(mode, P, G, weights, cfg, dev=local_rank, path=-1)
            auto = r_auto["engine_path"]
            other = 1 if auto == 2 else 2
            runs = {auto: r_auto, other: run_bs1(mode, P, G, weights, cfg, dev=local_rank, path=other)}
            r = dict(runs[auto])
            r["path"] = names[auto] + " (automatic)"
            r["roofline_frac"] = round(r["achieved_gbs"] / peak, 4)
            r["paths_tok_s"] = {names[k]: round(v["tok_s"], 2) for k, v in runs.items()}
            line[f"bs1_{mode}"] = r
        # opt-in INT8 tied lm_head (not reference-identical): the fastest path of the INT8 model
        r = run_bs1("int8", 512, 512, weights, cfg, dev=local_rank, path=2, lm8=True)
        line["bs1_int8_lm8"] = {"tok_s": round(r["tok_s"], 2), "ms_per_token": round(r["ms_per_token"], 4),
                                "bytes_per_token": r["bytes_per_token"],
                                "roofline_frac": round(r["achieved_gbs"] / peak, 4),
                                "note": "opt-in INT8 lm_head (vb_engine_quantize_lm_head); logits differ from "
                                        "the reference's by the lm_head quantisation"}
        line["gemv"] = gemv_microbench(local_rank)
        line["attn_sweep"] = attn_microbench(local_rank)
    if grp.rank == 0 and N == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg, weights, args)
    grp.close()
    if grp.rank == 0:
        print(json.dumps(line), flush=True)


def cpu_baseline(cfg, weights, args):
    import oracle
    if not oracle.have_ref():
        return {"value": None, "unit": "tok/s", "kind": "reference",
                "sample": "oracle/_ref not built"}
    procs = ref_procs()
    with tempfile.TemporaryDirectory() as td:
        mdir = write_model(td, cfg, weights)
        rate, secs = ref_time(mdir, "int8", args.prompt, 1, 3, procs)
        out = {"value": round(rate, 4), "unit": "tok/s", "cores": procs, "kind": "reference",
               "sample": f"reference Model::step (oracle/_ref), INT8, context {args.prompt}, "
                         f"{procs} single-threaded processes x 3 timed decode steps "
                         f"(+1 warm-up), one sequence each",
               "cpu": cpu_model(), "nproc": os.cpu_count(),
               "step_s_median": round(statistics.median(secs), 3)}
        if not args.no_extras:
            r32, s32 = ref_time(mdir, "f32", 32 + 64, 0, 2, 1)
            r8, s8 = ref_time(mdir, "int8", 512 + 256, 0, 2, 1)
            out["bs1_f32"] = {"value": round(r32, 4), "cores": 1,
                              "sample": "2 decode steps at context 96 (config 1 mid-point)"}
            out["bs1_int8"] = {"value": round(r8, 4), "cores": 1,
                               "sample": "2 decode steps at context 768 (config 3 mid-point)"}
    return out


def reference_weights(cfg):
    """The benchmark's weights drawn by the oracle's copy of the generator: the
    reference arm never loads the engine library."""
    import oracle
    import vbsynth
    return vbsynth.make_weights(cfg, seed=WEIGHT_SEED, normal=oracle.synth_normal)


def main_reference(args, rank, world):
    """Reference arm: the reference's own CPU decode (oracle/_ref, Model::step
    compiled from its sources) on this host's cores, same metric and workload
    config as the engine's line.  One step = one decode token of each of P
    single-threaded reference processes (the engine has no batching), each at
    the workload's context length; K timed steps after W warm-up steps."""
    if rank != 0:
        return 0
    import oracle
    import vbsynth
    if not oracle.have_ref():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libverbum_ref.so not built"}))
        return 0
    cfg = vbsynth.qwen3_config()
    weights = reference_weights(cfg)
    procs = ref_procs()
    K, W = args.steps, args.warmup
    with tempfile.TemporaryDirectory() as td:
        mdir = write_model(td, cfg, weights)
        del weights
        rate, secs = ref_time(mdir, "int8", args.prompt, W, K, procs)
    sample = (f"reference Model::step (oracle/_ref, compiled from the reference sources), INT8 "
              f"projections + f32 lm_head, context {args.prompt}: {procs} single-threaded "
              f"processes, one sequence each; a step is one decode token of every process")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(rate, 4), "unit": "tok/s",
        "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(1e3 * statistics.mean(secs), 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) random-init weights, uniform random prompt ids",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": procs,
                         "kind": "reference", "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
