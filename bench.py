"""Benchmark: one rubidium-train training step (forward + backward + fused
Adam tail) per step on synthetic data, through librbk's sm_100a kernels.

Default workload (N=1): the GPT-2-small-shaped decoder — 12 layers, d=768,
12 heads, FFN 3072 (GELU), vocab 50257, seq 1024, micro-batch 16 per GPU,
FP16 activations / FP32 masters, dynamic loss scale from 65536, per-layer
activation checkpointing, random init N(0, 0.02), uniform random tokens.
With --gpus N (torchrun, one rank per GPU) the same per-GPU work runs data
parallel with bucketed (25 MB) NCCL all-reduce overlapped with the backward
("scaling": "weak").  --workload 1.3b selects the 1.3B decoder (24 x 2048,
16 heads, FFN 8192, seq 2048, micro-batch 8).

Printed by rank 0: one JSON line (see the keys below).  Timing: CUDA events
on the launching stream, barrier + synchronize around the timed region, max
over ranks.  Weights, activations and logits exceed the 126 MB L2, so no L2
flush is needed between steps.  --impl reference times the CPU restatement
of the same step (the reference's own engine cannot run a backward) on the
host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "rubidium-train_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "train tokens/s/GPU (fwd+bwd+Adam), backward ms/step, % of TC/HBM roofline"

WORKLOADS = {
    "gpt2-small": dict(cfg=dict(V=50257, T=1024, D=768, H=12, L=12, FF=3072), batch=16, seq=1024,
                       name="GPT-2-small decoder (L12 d768 H12 FF3072 V50257), seq 1024, micro-batch 16/GPU"),
    "1.3b": dict(cfg=dict(V=50257, T=2048, D=2048, H=16, L=24, FF=8192), batch=8, seq=2048,
                 name="1.3B decoder (L24 d2048 H16 FF8192 V50257), seq 2048, micro-batch 8/GPU"),
    "tiny": dict(cfg=dict(V=4096, T=128, D=256, H=4, L=4, FF=1024), batch=8, seq=128,
                 name="tiny decoder (L4 d256 H4 FF1024 V4096), seq 128, batch 8"),
    # LoRA fine-tune of the GPT-2-small base: frozen FP16 base, rank-16 adapters on Q and V
    # (A ~ N(0, 0.02), B = 0, alpha 32), gradients to A and B only; every 50th step +inf in 1 of
    # every 1e5 dlogits elements exercises the fused inf check and skipped step
    "lora": dict(cfg=dict(V=50257, T=1024, D=768, H=12, L=12, FF=3072), batch=32, seq=512,
                 lora=dict(rank=16, alpha=32.0), inject_every=50, inject_stride=100000,
                 name="LoRA r16 (Q, V; alpha 32) on the GPT-2-small base, seq 512, batch 32, "
                      "+inf in 1e-5 of dlogits every 50th step"),
}

CAT_NAMES = ["gemm", "attn_fwd", "attn_bwd", "ln_fwd", "ln_bwd", "softmax_xent", "adam_tail", "embedding", "other"]


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def mm_params(cfg):
    D, F, L, V = cfg["D"], cfg["FF"], cfg["L"], cfg["V"]
    return L * (4 * D * D + 2 * D * F) + V * D


def gemm_flops_per_step(cfg, ntok, ckpt=True, lora=False):
    """Algorithmic tensor-core FLOPs of the base GEMMs in one step: forward 2 P, backward
    4 P per token (2 P under LoRA: no weight gradients; P = matmul parameters), plus the
    checkpoint recompute of the QKV and W1 projections."""
    D, F, L = cfg["D"], cfg["FF"], cfg["L"]
    P = mm_params(cfg)
    rec = L * (3 * D * D + D * F) if ckpt else 0
    return 2.0 * ntok * ((2 if lora else 3) * P + rec)


def train_flops_per_token(cfg, seq, lora_rank=0):
    """6 P + 6 L T D (causal attention), recompute excluded (the published convention).  A
    LoRA step has no base weight gradients: 4 P + 6 L T D + 16 L D r (Q and V adapters)."""
    if lora_rank:
        return 4.0 * mm_params(cfg) + 6.0 * cfg["L"] * seq * cfg["D"] + 16.0 * cfg["L"] * cfg["D"] * lora_rank
    return 6.0 * mm_params(cfg) + 6.0 * cfg["L"] * seq * cfg["D"]


class Clocks:
    """nvidia-smi sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- CPU legs ----

# CPU sample per workload: one micro-batch-1 sequence of this many tokens (the workload's
# own sequence length where one step stays within about 10-30 s of host time).
CPU_SEQ = {"gpt2-small": 1024, "lora": 512, "1.3b": 256, "tiny": 128}


def cpu_threads():
    """Every core this process may run on (torchrun exports OMP_NUM_THREADS=1 to each rank,
    so the oracle's thread count is set explicitly)."""
    import oracle
    return oracle.set_threads()


def cpu_sample(workload, seq=None):
    """The CPU restatement (oracle) of one fwd+bwd+AdamW step of the same model
    at micro-batch 1 over `seq` tokens; returns (tokens/s, seconds, threads)."""
    import numpy as np
    import oracle
    wl = WORKLOADS[workload]
    cfg = dict(wl["cfg"])
    seq = seq or CPU_SEQ[workload]
    threads = cpu_threads()
    rng = np.random.default_rng(0)
    params = oracle.init_params(cfg, seed=1)
    tok = rng.integers(0, cfg["V"], seq).astype(np.int32)
    tgt = rng.integers(0, cfg["V"], seq).astype(np.int32)
    if wl.get("lora"):                                 # adapter gradients only, AdamW on the adapters
        r, alpha, D, L = wl["lora"]["rank"], wl["lora"]["alpha"], cfg["D"], cfg["L"]
        A = (0.02 * rng.standard_normal((2, L * D * r))).astype(np.float32)
        Bz = np.zeros((2, L * r * D), np.float32)
        t0 = time.perf_counter()
        _, dAq, dBq, dAv, dBv = oracle.model_lora_grad(cfg, params, A[0], Bz[0], A[1], Bz[1], r, alpha, tok, tgt,
                                                       1, seq)
        ad = np.concatenate([A.ravel(), Bz.ravel()])
        gd = np.concatenate([dAq, dAv, dBq, dBv]).astype(np.float32)
        oracle.adamw(ad, gd, np.zeros_like(ad), np.zeros_like(ad), 3e-4, 0.9, 0.999, 1e-8, 0.0, 1)
        dt = time.perf_counter() - t0
        return seq / dt, dt, threads
    m = np.zeros_like(params); v = np.zeros_like(params)
    t0 = time.perf_counter()
    _, g, _ = oracle.model_loss_grad(cfg, params, tok, tgt, 1, seq)
    oracle.adamw(params, g, m, v, 3e-4, 0.9, 0.999, 1e-8, 0.0, 1)
    dt = time.perf_counter() - t0
    return seq / dt, dt, threads


def reference_ops():
    """The reference's own CPU code (oracle/_ref/libref.so, compiled from its sources; it
    builds only without OpenMP, so one core): cpuops::layer_norm_backward, softmax_backward,
    cross_entropy_backward and adamw_step at the kernel-microbench shapes, and
    CPUTransformer::forward on one sequence of the tiny decoder with V = D (its LM head is only
    shape-correct then).  Inputs are staged first; only the reference call is timed."""
    import ctypes as C

    import numpy as np
    import oracle
    ref = oracle.ref_lib()
    if ref is None:
        return {"unavailable": "oracle/_ref/libref.so was not built (the reference tree was absent at build time)"}
    F = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))   # noqa: E731
    I = lambda a: a.ctypes.data_as(C.POINTER(C.c_int))     # noqa: E731
    rng = np.random.default_rng(0)
    out = {"kind": "reference", "cores": 1,
           "build": "g++ -O2 of src/cpu_mat.h + src/cpu_model.cpp without -fopenmp (oracle/Makefile target ref)"}
    # LayerNorm backward [16384, 1024] (src/cpu_mat.h:126-153)
    N, D = 16384, 1024
    x = rng.standard_normal((N, D), dtype=np.float32)
    dy = rng.standard_normal((N, D), dtype=np.float32)
    g = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    mean = x.mean(1).astype(np.float32)
    rstd = (1 / np.sqrt(x.var(1) + 1e-5)).astype(np.float32)
    s = ref.ref_time_layer_norm_backward(F(dy), F(x), F(g), F(mean), F(rstd), N, D)
    by = N * D * 6 + N * 8 + D * 10       # the same algorithmic bytes as the GPU kernel (FP16 sizes)
    out["layer_norm_backward_16384x1024"] = {"s": s, "GB/s": by / s / 1e9, "algorithmic_bytes": by}
    del x, dy
    # softmax backward over 8 * 16 * 1024 rows of 1024 (src/cpu_mat.h:190-200; it has no causal form)
    rows, T = 8 * 16 * 1024, 1024
    y = rng.random((rows, T), dtype=np.float32)
    dyy = rng.standard_normal((rows, T), dtype=np.float32)
    s = ref.ref_time_softmax_backward(F(dyy), F(y), rows, T)
    out["softmax_backward_B8H16T1024"] = {"s": s, "elements": rows * T, "Gelem/s": rows * T / s / 1e9}
    del y, dyy
    # cross-entropy backward [8192, 32000] (src/cpu_mat.h:220-236)
    N, V = 8192, 32000
    z = (2.0 * rng.standard_normal((N, V), dtype=np.float32))
    tg = rng.integers(0, V, N).astype(np.int32)
    s = ref.ref_time_cross_entropy_backward(F(z), I(tg), N, V)
    by = N * V * 4 + N * 4
    out["cross_entropy_backward_8192x32000"] = {"s": s, "GB/s": by / s / 1e9, "algorithmic_bytes": by}
    del z
    # AdamW over 16M parameters (src/cpu_mat.h:280-292)
    n = 1 << 24
    p = rng.standard_normal(n, dtype=np.float32)
    gg = rng.standard_normal(n, dtype=np.float32)
    s = ref.ref_time_adamw_step(F(p), F(gg), n, C.c_float(3e-4), C.c_float(0.9), C.c_float(0.999),
                                C.c_float(1e-8), C.c_float(0.01))
    out["adamw_step_16M"] = {"s": s, "params_per_s": n / s, "GB/s": 34.0 * n / s / 1e9}
    del p, gg
    # CPUTransformer::forward (src/cpu_model.cpp:115-222): the tiny decoder (L4 D256 H4 FF1024) with
    # V = D = 256, one sequence of 128 tokens, weights N(0, 0.02)
    cfg = dict(V=256, T=128, D=256, H=4, L=4, FF=1024)
    Vv, Tt, Dd, L, FF = cfg["V"], cfg["T"], cfg["D"], cfg["L"], cfg["FF"]
    w = lambda *sh: (0.02 * rng.standard_normal(sh)).astype(np.float32)   # noqa: E731
    blocks = []
    for _ in range(L):
        blocks += [np.ones(Dd), np.zeros(Dd), w(Dd, Dd), np.zeros(Dd), w(Dd, Dd), np.zeros(Dd), w(Dd, Dd),
                   np.zeros(Dd), w(Dd, Dd), np.zeros(Dd), np.ones(Dd), np.zeros(Dd), w(Dd, FF), np.zeros(FF),
                   w(FF, Dd), np.zeros(Dd)]
    layers = np.concatenate([np.asarray(b, np.float32).ravel() for b in blocks])
    tok = rng.integers(0, Vv, Tt).astype(np.int32)
    tgt = rng.integers(0, Vv, Tt).astype(np.int32)
    loss = C.c_float()
    ones, zeros = np.ones(Dd, np.float32), np.zeros(Dd, np.float32)
    te, pe, lw, lb = w(Vv, Dd), w(Tt, Dd), w(Dd, Vv), np.zeros(Vv, np.float32)
    s = ref.ref_time_cpu_forward(Vv, Tt, Dd, cfg["H"], L, FF, F(te), F(pe), F(layers), F(ones), F(zeros), F(lw),
                                 F(lb), I(tok), I(tgt), Tt, C.byref(loss))
    out["cpu_transformer_forward_tiny_v256"] = {"s": s, "tokens_per_s": Tt / s, "loss": loss.value,
                                                "config": "L4 D256 H4 FF1024 V256 T128, 1 sequence"}
    return out


def run_reference(args):
    """--impl reference: the CPU restatement of the step (the reference's own engine cannot run a
    backward) on every host core, plus the reference's own CPU ops timed serially."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    seq = CPU_SEQ[args.workload]
    vals, cores = [], 1
    budget_s, used = 90.0, 0.0
    for _ in range(min(args.warmup, 1)):
        cpu_sample(args.workload, seq)
    for i in range(args.steps):
        tps, dt, cores = cpu_sample(args.workload, seq)
        vals.append(tps)
        used += dt
        if used > budget_s:
            break
    v = statistics.median(vals)
    sample = (f"one fwd+bwd+AdamW{' (LoRA adapters)' if wl.get('lora') else ''} step of the same model over "
              f"1 x {seq} tokens per timed step (oracle, {cores} threads)")
    out = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": len(vals), "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * seq / v, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": wl["name"] + f"; CPU sample: micro-batch 1 x {seq} tokens per step",
                   "value_scope": "whole host (all cores of the node)"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload != "tiny" and not args.no_ref_ops:
        out["cpu_baseline"]["reference_ops"] = reference_ops()
    print(json.dumps(out), flush=True)
    return 0


# ------------------------------------------------------------- microbench ----

def graph_time(torch, fn, n):
    """ms per call of fn(i), i = 0..n-1, from one replay of a CUDA graph holding the n calls, so the
    host's per-call cost (ctypes, launch) does not pace kernels of a few tens of microseconds.  Three
    eager warm-up calls first; an eager loop if the calls cannot be captured."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                for i in range(n):
                    fn(i)
        torch.cuda.current_stream().wait_stream(side)
        graph.replay()                                  # warm
        torch.cuda.synchronize()
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        del graph
        return s.elapsed_time(e) / n
    except RuntimeError:
        torch.cuda.synchronize()
    s.record()
    for i in range(n):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / n


def microbench(ops, torch, hbm_peak, reps=20):
    """HBM-bound backward kernels at their configured shapes (GB/s of algorithmic bytes)."""
    res = {}
    dev = "cuda"

    def timeit(fn, n=reps):
        return graph_time(torch, fn, n)

    g = torch.Generator(device=dev).manual_seed(0)
    # (a) LN backward [16384, 1024]: 4 input sets rotate so the 64 MB per set is not L2-resident
    N, D = 16384, 1024
    sets = []
    for k in range(4):
        x = torch.randn(N, D, device=dev, generator=g).half()
        dy = torch.randn(N, D, device=dev, generator=g).half()
        sets.append((x, dy))
    gam = (1 + 0.02 * torch.randn(D, device=dev, generator=g)).half()
    mean = torch.empty(N, device=dev); rstd = torch.empty(N, device=dev)
    _, mean, rstd = ops.ln_fwd(sets[0][0], gam, torch.zeros(D, device=dev).half())
    dx = torch.empty(N, D, device=dev, dtype=torch.float16)
    dg = torch.zeros(D, device=dev); db = torch.zeros(D, device=dev)
    C = ops.ctx()
    import ctypes
    from rbk._lib import call

    def ln(i):
        x, dy = sets[i % 4]
        call("rbk_ln_bwd", C.handle, ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(dg.data_ptr()),
             ctypes.c_void_p(db.data_ptr()), None, ctypes.c_void_p(dy.data_ptr()), None,
             ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(gam.data_ptr()), ctypes.c_void_p(mean.data_ptr()),
             ctypes.c_void_p(rstd.data_ptr()), N, D, 0, ops._s())
    ms = timeit(ln)
    by = N * D * 6 + N * 8 + D * 10
    res["ln_bwd_16384x1024"] = {"ms": ms, "GB/s": by / ms / 1e6, "frac_of_hbm": by / ms / 1e6 / hbm_peak,
                                "algorithmic_bytes": by}
    del sets
    # (b) softmax-CE backward [8192, 32000] FP16 logits ~N(0,2), uniform targets (524 MB in, 524 MB out)
    N, V = 8192, 32000
    z = (2.0 * torch.randn(N, V, device=dev, generator=g)).half()
    t = torch.randint(0, V, (N,), device=dev, generator=g, dtype=torch.int32)
    d = torch.empty_like(z)

    def ce(i):
        call("rbk_softmax_xent_bwd", C.handle, ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(z.data_ptr()), V,
             ctypes.c_void_p(t.data_ptr()), N, V, ctypes.c_float(65536.0 / N), None, None, ops._s())
    ms = timeit(ce)
    by = N * V * 4 + N * 4
    res["softmax_xent_bwd_8192x32000"] = {"ms": ms, "GB/s": by / ms / 1e6, "frac_of_hbm": by / ms / 1e6 / hbm_peak,
                                          "algorithmic_bytes": by}
    del z, d
    # (c) causal attention-softmax backward B8 H16 T1024 (P, dP in, dS out over the lower triangle)
    nm, T = 8 * 16, 1024
    P = torch.rand(nm, T, T, device=dev, generator=g).half()
    dP = torch.randn(nm, T, T, device=dev, generator=g).half()
    dS = torch.empty_like(P)

    def sm(i):
        call("rbk_attn_softmax_bwd", C.handle, ctypes.c_void_p(dS.data_ptr()), ctypes.c_void_p(P.data_ptr()),
             ctypes.c_void_p(dP.data_ptr()), nm, T, 1, ops._s())
    ms = timeit(sm)
    by = nm * T * (T + 1) // 2 * 6
    res["attn_softmax_bwd_B8H16T1024"] = {"ms": ms, "GB/s": by / ms / 1e6, "frac_of_hbm": by / ms / 1e6 / hbm_peak,
                                          "algorithmic_bytes": by}
    del P, dP, dS
    torch.cuda.empty_cache()
    return res


def tokenizer_bench(torch, hbm_peak, cpu=True):
    """The GPU BPE tokenizer (rbk_bpe_*, the data path of src/tokenizer_cuda.cu:90-203) on a
    GPT-2-sized synthetic tokenizer (50257 ids, 49996 rules; seeded Zipf text, no dataset offline):
      encode_2048: 16384 strings x 2047 bytes -> rows of 2048 tokens, inputs resident (value) and
                   from host strings through rbk_bpe_encode_batch (e2e: packing + H2D + kernel);
      encode_256:  65536 strings x 254 bytes at max_seq_len 256, the reference kernel's domain (one
                   block of 256 threads per string), with the reference's own algorithm (its kernels
                   compiled for the CPU, serial) and the oracle port timed on bounded samples;
      decode_2048: the encode_2048 rows back to strings of up to 4096 bytes.
    Algorithmic bytes: text + offsets (8) + lengths (4) in, rows (4 x max_seq_len) + lengths (4) out."""
    import numpy as np

    import oracle
    from rbk.tokenizer import GPUTokenizer, pack_strings, synthetic_batch, synthetic_corpus, synthetic_tables
    vocab, merges, words = synthetic_tables()
    corpus = synthetic_corpus(words, 1 << 25, seed=9)
    tk = GPUTokenizer(vocab, merges)
    res = {"tokenizer": "synthetic GPT-2-sized: 50257 ids, %d rules, Zipf(1.1) pseudo-words" % tk.num_rules}
    st = torch.cuda.current_stream()

    def dev_time(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        for _ in range(n):
            fn()
        e.record(st)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n

    for name, B, L, ms in (("encode_2048", 16384, 2047, 2048), ("encode_256", 65536, 254, 256)):
        strs = synthetic_batch(corpus, B, L, seed=4)
        data, offs, lens = pack_strings(strs)
        d_data, d_offs, d_lens = (torch.from_numpy(a.copy()).cuda() for a in (data, offs, lens))
        rows = torch.empty(B, ms, dtype=torch.int32, device="cuda")
        rl = torch.empty(B, dtype=torch.int32, device="cuda")
        ms_launch = dev_time(lambda: tk.encode(d_data, d_offs, d_lens, ms, out=rows, out_lengths=rl), 10)
        n_tok = int(rl.sum().item()) - B
        by = data.size + 12 * B + 4 * B * ms + 4 * B
        gbs = by / ms_launch / 1e6
        ent = {"strings": B, "bytes_per_string": L, "max_seq_len": ms, "ms_per_launch": ms_launch,
               "text_MB_per_s": data.size / ms_launch / 1e3, "tokens_per_s": n_tok / ms_launch * 1e3,
               "strings_per_s": B / ms_launch * 1e3, "tokens_per_string": n_tok / B,
               "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                            "frac": gbs / hbm_peak, "algorithmic_bytes_per_launch": by,
                            "note": "the pair lookups hit L1/L2 (a 4 MB table); DRAM carries only text in and rows out"}}
        if name == "encode_2048":
            # e2e: host strings -> device rows through the reference-facing entry (the char** a C
            # caller holds; building it from Python objects is timed separately), lengths read back
            from rbk.tokenizer import host_strings
            t0 = time.perf_counter()
            arr = host_strings(strs)
            py_ms = (time.perf_counter() - t0) * 1e3
            for _ in range(2):
                tk.encode_batch(arr, ms, out=rows, out_lengths=rl)
            torch.cuda.synchronize()
            reps = 5
            t0 = time.perf_counter()
            for _ in range(reps):
                tk.encode_batch(arr, ms, out=rows, out_lengths=rl)
                lh = rl.cpu()
            dt = (time.perf_counter() - t0) / reps
            ent["e2e"] = {"text_MB_per_s": data.size / dt / 1e6, "strings_per_s": B / dt, "ms_per_call": dt * 1e3,
                          "h2d_bytes_per_call": int(data.size + 12 * B), "d2h_bytes_per_call": int(lh.numel() * 4),
                          "path": "rbk_bpe_encode_batch (host strings: lengths and packing into pinned staging "
                                  "on up to 8 threads, in four parts whose H2D copies and encode launches "
                                  "overlap the packing of the next) + lengths D2H, per call",
                          "python_char_array_ms": py_ms}
            # decode the rows back
            out = torch.empty(B, 4096, dtype=torch.uint8, device="cuda")
            ms_dec = dev_time(lambda: tk.decode_batch(rows, rl, 4096, out=out), 10)
            dby = 4 * (n_tok + B) + 4 * B + data.size + B   # tokens read up to the EOS, text + NULs written
            ent_dec = {"strings": B, "ms_per_launch": ms_dec, "text_MB_per_s": data.size / ms_dec / 1e3,
                       "roofline": {"bound": "hbm", "achieved": dby / ms_dec / 1e6, "peak": hbm_peak, "unit": "GB/s",
                                    "frac": dby / ms_dec / 1e6 / hbm_peak, "algorithmic_bytes_per_launch": dby}}
            ok = bytes(out[7].cpu().numpy()).split(b"\0", 1)[0] == strs[7]
            ent_dec["round_trip_row7"] = bool(ok)
            res["decode_2048"] = ent_dec
            del out
        if cpu:
            # oracle port (hash-map restatement) on bounded samples: one thread, then every core
            # (strings in parallel); its rows are checked against the GPU's
            k = 2048 if ms == 2048 else 16384
            sd, so, sl = pack_strings(strs[:k])
            oracle.set_threads(1)
            t0 = time.perf_counter()
            orow, orl, _ = oracle.bpe_encode(merges, sd, so, sl, ms)
            dt = time.perf_counter() - t0
            same = bool(np.array_equal(orl, rl[:k].cpu().numpy()) and np.array_equal(orow, rows[:k].cpu().numpy()))
            ent["cpu_baseline_port"] = {"value": sd.size / dt / 1e6, "unit": "text MB/s", "cores": 1, "kind": "port",
                                        "sample": f"first {k} strings", "rows_equal_gpu": same}
            cores = cpu_threads()
            sd, so, sl = pack_strings(strs)
            t0 = time.perf_counter()
            oracle.bpe_encode(merges, sd, so, sl, ms)
            dt = time.perf_counter() - t0
            ent["cpu_baseline_port_all_cores"] = {"value": sd.size / dt / 1e6, "unit": "text MB/s", "cores": cores,
                                                  "kind": "port", "sample": f"all {B} strings ({dt:.1f} s)"}
            if ms == 256 and oracle.reftok_lib() is not None:
                kr = 256
                sd, so, sl = pack_strings(strs[:kr])
                dt = oracle.ref_bpe_time_encode(merges, sd, so, sl, ms, 1)
                ent["cpu_baseline_reference"] = {
                    "value": sd.size / dt / 1e6, "unit": "text MB/s", "cores": 1, "kind": "reference",
                    "sample": f"first {kr} strings ({dt:.1f} s)",
                    "note": "encode_kernel's algorithm (thread 0 merges serially, find_merge scans every rule "
                            "per pair) compiled for the CPU; on a GPU it runs the same loop on one thread per block"}
        res[name] = ent
        del d_data, d_offs, d_lens, rows, rl
    tk.close()
    torch.cuda.empty_cache()
    return res


def r8(x):
    return (x + 7) // 8 * 8


def gemm_shapes(N=16384, D=768, F=3072, V=50257, prefix="gemm"):
    """The GEMMs of one GPT-2-small layer step and the LM head, as the model issues them:
    name -> (M, N, K, a_major, b_major, epilogue, extra) with extra in {"", "bias", "res", "dbias"}."""
    s = {
        "fwd_qkv": (N, 3 * D, D, 0, 0, 0, "bias"),
        "fwd_wo": (N, D, D, 0, 0, 0, "res"),
        "fwd_w1": (N, F, D, 0, 0, 1, "bias"),
        "fwd_w2": (N, D, F, 0, 0, 0, "res"),
        "lm_fwd": (N, V, D, 0, 0, 0, "bias"),
        "dgrad_lm": (N, D, V, 0, 1, 0, ""),
        "wgrad_lm": (V, D, N, 1, 1, 3, "dbias"),
        "wgrad_w2": (D, F, N, 1, 1, 3, ""),
        "dgrad_w2": (N, F, D, 0, 1, 2, ""),
        "wgrad_w1": (F, D, N, 1, 1, 3, "dbias"),
        "dgrad_w1": (N, D, F, 0, 1, 0, ""),
        "wgrad_wo": (D, D, N, 1, 1, 3, ""),
        "dgrad_wo": (N, D, D, 0, 1, 0, ""),
        "wgrad_qkv": (3 * D, D, N, 1, 1, 3, ""),
        "dgrad_qkv": (N, D, 3 * D, 0, 1, 0, ""),
    }
    return {f"{prefix}_{k}": v for k, v in s.items()}


def all_gemm_shapes():
    """GPT-2-small shapes as gemm_*, the 1.3B decoder's (N = 8 x 2048, D 2048, FF 8192) as gemm13_*."""
    out = gemm_shapes()
    out.update(gemm_shapes(16384, 2048, 8192, 50257, prefix="gemm13"))
    return out


def gemm_case(name, torch, ops, g):
    """(launch function, FLOPs per launch) of one step GEMM shape; inputs rotate over enough sets
    (> 2x the 126 MB L2) that every launch reads them from DRAM."""
    shapes = all_gemm_shapes()
    if name not in shapes:
        raise SystemExit(f"unknown GEMM {name}: one of {sorted(shapes)}")
    M, Nn, K, am, bm, epi, extra = shapes[name]
    lda, ldb, ldc = r8(M if am else K), r8(Nn if bm else K), r8(Nn)
    f32 = epi in (ops.EPI_ACC_F32, ops.EPI_STORE_F32)
    set_bytes = 2 * ((K if am else M) * lda + (K if bm else Nn) * ldb) + M * ldc * (4 if f32 else 2) * \
        (2 if epi in (ops.EPI_GELU_BWD, ops.EPI_BIAS_GELU) or extra == "res" else 1)
    nsets = max(1, min(16, -(-300_000_000 // set_bytes)))
    sets = []
    for _ in range(nsets):
        A = (0.5 * torch.randn(K if am else M, lda, device="cuda", generator=g)).half()
        B = (0.5 * torch.randn(K if bm else Nn, ldb, device="cuda", generator=g)).half()
        Cm = torch.zeros(M, ldc, device="cuda", dtype=torch.float32 if f32 else torch.float16)
        aux = torch.randn(M, ldc, device="cuda", generator=g).half() \
            if epi == ops.EPI_GELU_BWD or extra == "res" else None
        aux_out = torch.empty(M, ldc, device="cuda", dtype=torch.float16) if epi == ops.EPI_BIAS_GELU else None
        sets.append((A, B, Cm, aux, aux_out))
    bias = torch.randn(ldc, device="cuda", generator=g).half() if extra == "bias" or epi == ops.EPI_BIAS_GELU \
        else None
    dbias = torch.zeros(M, device="cuda") if extra == "dbias" else None
    it = [0]

    def fn():
        A, B, Cm, aux, aux_out = sets[it[0] % nsets]
        it[0] += 1
        ops.gemm(A, B, M, Nn, K, am, bm, C_out=Cm, ldc=ldc, epilogue=epi, bias=bias, aux=aux, aux_out=aux_out,
                 dbias_rows=dbias, lda=lda, ldb=ldb, store_c=epi != ops.EPI_BIAS_GELU)
    return fn, 2.0 * M * Nn * K


def kernel_loop(name, reps, torch, ops):
    """One kernel at a representative GPT-2-small shape, `reps` launches (for ncu
    captures and tuning).  Prints per-launch time and the achieved rate.  GEMM inputs
    rotate over enough sets (> 2x the 126 MB L2) that every launch reads them from DRAM.
    gemm_all: every GEMM shape of the step in turn (no timing line)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    hbm, tc, tcs, _ = peaks()
    N, D, F, V = 16384, 768, 3072, 50257
    if name == "gemm_all":
        # every GEMM shape of the GPT-2-small step, `reps` launches each, one shape resident at a
        # time (for one ncu capture of their DRAM traffic)
        for k in gemm_shapes():
            fn, _ = gemm_case(k, torch, ops, g)
            for _ in range(reps):
                fn()
            torch.cuda.synchronize()
            del fn
            torch.cuda.empty_cache()
        print(json.dumps({"kernel": name, "shapes": len(gemm_shapes()), "launches_each": reps}), flush=True)
        return 0
    if name.startswith("gemm"):
        fn, work = gemm_case(name, torch, ops, g)
        unit, peak = "TFLOP/s", tc
    elif name == "ln_bwd" or name.startswith("ln_bwd_"):
        # ln_bwd: [16384, 1024]; ln_bwd_<D>: 2^24 elements of width D.  Four input sets (256 MB)
        # rotate, so x and dy come from DRAM as in the step.
        Dl = int(name[7:]) if name != "ln_bwd" else 1024
        Nl = ((1 << 24) // Dl) // 4 * 4
        sets = [(torch.randn(Nl, Dl, device="cuda", generator=g).half(),
                 torch.randn(Nl, Dl, device="cuda", generator=g).half()) for _ in range(4)]
        gam = (1 + 0.02 * torch.randn(Dl, device="cuda", generator=g)).half()
        _, mean, rstd = ops.ln_fwd(sets[0][0], gam, torch.zeros(Dl, device="cuda").half())
        dgam, dbet = torch.zeros(Dl, device="cuda"), torch.zeros(Dl, device="cuda")
        it = [0]

        def fn():
            x, dy = sets[it[0] % 4]
            it[0] += 1
            ops.ln_bwd(dy, x, gam, mean, rstd, dgamma=dgam, dbeta=dbet)
        work, unit, peak = Nl * Dl * 6 + Nl * 8 + Dl * 10, "GB/s", hbm
    elif name.startswith("ln_fwd_"):
        # LayerNorm forward over 2^24 elements of width D, four input sets rotating (256 MB)
        Dl = int(name[7:])
        Nl = ((1 << 24) // Dl) // 4 * 4
        xs = [torch.randn(Nl, Dl, device="cuda", generator=g).half() for _ in range(4)]
        gam = (1 + 0.02 * torch.randn(Dl, device="cuda", generator=g)).half()
        bet = (0.02 * torch.randn(Dl, device="cuda", generator=g)).half()
        it = [0]

        def fn():
            ops.ln_fwd(xs[it[0] % 4], gam, bet)
            it[0] += 1
        work, unit, peak = Nl * Dl * 4 + Nl * 8 + Dl * 4, "GB/s", hbm
    elif name == "xent":
        z = (2 * torch.randn(8192, 32000, device="cuda", generator=g)).half()
        t = torch.randint(0, 32000, (8192,), device="cuda", dtype=torch.int32, generator=g)

        def fn():
            ops.softmax_xent_bwd(z, t, scale=8.0, out=z, want_loss=False)
        work, unit, peak = 8192 * 32000 * 4 + 8192 * 4, "GB/s", hbm
    elif name in ("attn_fwd", "attn_bwd"):
        qkv = (0.5 * torch.randn(N, 3 * D, device="cuda", generator=g)).half()
        o, lse = ops.attn_fwd(qkv, 16, 1024, 12, 64)
        do = torch.randn(N, D, device="cuda", generator=g).half()
        tri = 16 * 12 * 1024 * 1025 / 2 * 64

        def fn():
            if name == "attn_fwd":
                ops.attn_fwd(qkv, 16, 1024, 12, 64)
            else:
                ops.attn_bwd(qkv, o, do, lse, 16, 1024, 12, 64)
        work, unit, peak = (4 if name == "attn_fwd" else 8) * tri, "TFLOP/s", tc
    elif name == "adam_tail":
        n = 163_000_000 // 64 * 64
        p, gr, m, v = (torch.zeros(n, device="cuda") for _ in range(4))
        p16 = torch.empty(n, device="cuda", dtype=torch.float16)
        sc = ops.new_scaler()

        def fn():
            ops.adam_tail(p, gr, m, v, p16, sc, lr=1e-4)
        work, unit, peak = 34.0 * n, "GB/s", hbm
    elif name in ("bpe_encode", "bpe_encode_256", "bpe_decode"):
        # the GPU tokenizer: 16384 strings x 2047 bytes of synthetic text -> rows of 2048 tokens
        # (33 MB in, 134 MB out), or 65536 x 254 bytes -> rows of 256 (bpe_encode_256, one warp
        # per string), GPT-2-sized synthetic rule table; decode turns the 2048-token rows back
        from rbk.tokenizer import GPUTokenizer, pack_strings, synthetic_batch, synthetic_corpus, synthetic_tables
        vocab, merges, words = synthetic_tables()
        tk = GPUTokenizer(vocab, merges)
        B, L, ms = (65536, 254, 256) if name == "bpe_encode_256" else (16384, 2047, 2048)
        strs = synthetic_batch(synthetic_corpus(words, 1 << 25, seed=9), B, L, seed=4)
        data, offs, lens = pack_strings(strs)
        dd, do, dl = (torch.from_numpy(a.copy()).cuda() for a in (data, offs, lens))
        rows = torch.empty(B, ms, dtype=torch.int32, device="cuda")
        rl = torch.empty(B, dtype=torch.int32, device="cuda")
        tk.encode(dd, do, dl, ms, out=rows, out_lengths=rl)
        sout = torch.empty(B, 4096, dtype=torch.uint8, device="cuda") if name == "bpe_decode" else None

        def fn():
            if name == "bpe_decode":
                tk.decode_batch(rows, rl, 4096, out=sout)
            else:
                tk.encode(dd, do, dl, ms, out=rows, out_lengths=rl)
        # algorithmic bytes: text + offsets + lengths in, full rows + lengths out (encode); tokens up
        # to the EOS + lengths in, text + NULs out (decode)
        work = data.size + B * (12 + 4 * ms + 4) if name != "bpe_decode" else \
            4 * int(rl.sum().item()) + B * 5 + data.size
        unit, peak = "GB/s", hbm
    else:
        raise SystemExit(f"unknown kernel {name}")
    if os.environ.get("RBK_BENCH_EAGER") == "1" or name.startswith("attn") or name == "adam_tail" or \
            name.startswith("bpe_"):
        for _ in range(3):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / reps
    else:
        ms = graph_time(torch, lambda i: fn(), reps)
    rate = work / (ms * 1e-3) / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"kernel": name, "ms_per_launch": ms, "achieved": rate, "unit": unit, "peak": peak,
                      "frac": rate / peak}), flush=True)
    return 0


# ------------------------------------------------------------------ GPU leg ----

# Mean DRAM read + write bytes of one GEMM launch of the GPT-2-small step: every GEMM shape
# of the step captured alone with ncu (dram__bytes_read.sum + dram__bytes_write.sum, inputs
# rotating over more than L2), weighted by that shape's launches per step (171).  The per-shape
# figures and the command are in profiles/gemm_shapes_dram.md.
GEMM_TRAFFIC_PER_LAUNCH = 141.3e6


def check_dp(model, tokens, targets, B, S, world, dist, torch):
    """Cross-rank check of the data-parallel gradients at this world size, on the workload's
    own model: (1) two micro-steps without all-reduce give this rank's local sum L; (2) the
    same two micro-steps with the second all-reducing (gradient accumulation) give G.  G must
    equal the plain sum over ranks of L (an independent NCCL all-reduce of L) and be
    bit-identical on every rank (a checksum of its bits, gathered).  Under the sharded optimizer
    each rank holds the sum on its own slices only (the rest is zero): G is compared there, and
    the ranks must agree bit for bit on the weights after one optimizer step."""
    g2 = torch.roll(targets, 1, dims=1)               # a second micro-batch
    model.grad.zero_()
    with model.no_sync():
        for t in (targets, g2):
            model.forward(tokens, t, B, S)
            model.backward(tokens, t, B, S, 0.5)
    local = model.grad.clone()
    model.grad.zero_()
    with model.no_sync():
        model.forward(tokens, targets, B, S)
        model.backward(tokens, targets, B, S, 0.5)
    model.forward(tokens, g2, B, S)
    model.backward(tokens, g2, B, S, 0.5)
    torch.cuda.synchronize()
    G = model.grad
    dist.all_reduce(local, op=dist.ReduceOp.SUM)
    ranges = model.dp_shard_ranges()
    if ranges:
        own = torch.zeros(G.numel(), dtype=torch.bool, device=G.device)
        for b, e in ranges:
            own[b:e] = True
        err2 = torch.stack([((G - local) * own).norm() ** 2, (local * own).norm() ** 2])
        dist.all_reduce(err2, op=dist.ReduceOp.SUM)       # over the union of the slices: the arena
        rel = float(err2[0].sqrt() / err2[1].sqrt().clamp_min(1e-30))
        finite = bool(torch.isfinite(G).all()) and int(torch.count_nonzero(G * ~own)) == 0
        model.optimizer_step(0, 1e-4)
        model.dp_gather_state()
        torch.cuda.synchronize()
        what = torch.cat([model.p16.view(torch.int16).to(torch.int32), model.p32.view(torch.int32)])
        del own
    else:
        rel = float((G - local).norm() / local.norm().clamp_min(1e-30))
        finite = bool(torch.isfinite(G).all())
        what = G.view(torch.int32)
    bits = what.to(torch.int64)
    idx = torch.arange(bits.numel(), device=bits.device, dtype=torch.int64) % 1000003 + 1
    cs = torch.stack([(bits * idx).sum(), bits.sum()])
    allcs = [torch.zeros_like(cs) for _ in range(world)]
    dist.all_gather(allcs, cs)
    agree = all(bool(torch.equal(c, allcs[0])) for c in allcs)
    model.grad.zero_()
    del local, bits, idx, what
    torch.cuda.synchronize()
    # tolerance: two backwards of the same inputs differ by FP32 accumulation-order noise that FP16
    # roundings carry forward (measured ~2e-4); the schedule error this guards against is O(1)
    return {"ga": 2, "ranks_bitwise_equal": agree, "checksum": int(allcs[0][0]), "finite": finite,
            "rel_l2_vs_allreduce_of_local_sums": rel, "tolerance": 2e-3, "ok": agree and finite and rel < 2e-3,
            "sharded_optimizer": bool(ranges),
            "how": "grad after 2 micro-steps (the 1st without all-reduce) vs an independent all-reduce "
                   "of each rank's 2-micro-step local sum (sharded: on each rank's slices); bit checksums "
                   "gathered from every rank (sharded: of the FP16 and FP32 weights after one optimizer step)"}


def run_workload(name, args, world, rank, local, dist, torch, steps, warmup, e2e=True, profile=True,
                 dp_check=False):
    """Builds the workload's model, times `steps` training steps after `warmup`, then a profiled
    pass (per-launch events) and an end-to-end pass.  Returns the result dict (rank 0 prints)."""
    import ctypes

    from rbk import lib
    from rbk.model import ModelConfig, RubidiumTransformer, dp_unique_id

    hbm_peak, tc_burst, tc_sustained, peak_kind = peaks()
    wl = WORKLOADS[name]
    cfg = wl["cfg"]
    B, S = wl["batch"], wl["seq"]
    ntok = B * S
    ckpt = not args.no_ckpt
    model = RubidiumTransformer(ModelConfig(**cfg, use_activation_checkpointing=ckpt), max_batch=B, max_seq=S)
    model.init_weights(seed=42, std=0.02)
    lora = wl.get("lora")
    if lora:
        model.init_lora(rank=lora["rank"], alpha=lora["alpha"])
    if world > 1:
        uid = [dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.dp_init(rank, world, uid[0], int(args.bucket_mb * (1 << 20)), shard=args.dp_shard and not lora)

    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    tokens = torch.randint(0, cfg["V"], (B, S), device="cuda", dtype=torch.int32, generator=g)
    targets = torch.randint(0, cfg["V"], (B, S), device="cuda", dtype=torch.int32, generator=g)
    stream = torch.cuda.current_stream()

    nstep = [0]   # steps run so far (warm-up included): the LoRA workload injects on every 50th

    def backward(tok, tgt):
        nstep[0] += 1
        if lora and nstep[0] % wl["inject_every"] == 0:
            model.inject_inf(offset=nstep[0] % wl["inject_stride"], stride=wl["inject_stride"])
        model.backward(tok, tgt, B, S, 1.0)

    def update():
        if lora:
            model.lora_optimizer_step(0, 3e-4, 0.9, 0.999, 1e-8, 0.0)
        else:
            model.optimizer_step(0, 3e-4, 0.9, 0.999, 1e-8, 0.0)

    def step():
        model.forward(tokens, targets, B, S)
        backward(tokens, targets)
        update()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()

    # ---------------- timed region (device events, max over ranks) ----------
    # The headline pass records no per-kernel events (they cost ~4% of the step and
    # break launch overlap); a second pass of the same steps with an event pair around
    # every launch gives the per-kernel split and the GEMM roofline.
    mctx = ctypes.c_void_p()
    lib().rbk_model_ctx(model.handle, ctypes.byref(mctx))
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.5)   # let the sampler come up before the timed region
    bw_s = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    bw_e = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    launches0 = lib().rbk_launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(steps):
        model.forward(tokens, targets, B, S)
        bw_s[i].record(stream)
        backward(tokens, targets)
        bw_e[i].record(stream)
        update()
    t_end.record(stream)
    torch.cuda.synchronize()
    launches = lib().rbk_launch_count() - launches0
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end)
    bwd_ms = statistics.median(bw_s[i].elapsed_time(bw_e[i]) for i in range(steps))
    if world > 1:
        t = torch.tensor([ms, bwd_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, bwd_ms = float(t[0]), float(t[1])
    ms_step = ms / steps
    res = {"workload": wl["name"], "value": world * ntok / (ms_step / 1000.0), "unit": "tokens/s",
           "tokens_per_s_per_gpu": ntok / (ms_step / 1000.0), "ms_per_step": ms_step, "steps": steps,
           "warmup": warmup, "backward_ms_per_step": bwd_ms, "gpu_launches": int(launches), "clocks": clk,
           "global_batch": B * world, "seq_len": S, "activation_checkpointing": ckpt,
           "train_tflops_per_gpu": train_flops_per_token(cfg, S, lora["rank"] if lora else 0) * ntok /
                                   (ms_step / 1000.0) / 1e12,
           "gemm_flops_per_step": gemm_flops_per_step(cfg, ntok, ckpt, bool(lora))}
    if world > 1:
        res["allreduce_bytes_per_step"] = 4 * (model.lora_tensors("grad")[0].numel() * 4 if lora else model.nparams)
        res["sharded_optimizer"] = bool(args.dp_shard and not lora)
        if res["sharded_optimizer"]:   # FP32 gradients reduce-scattered, FP16 weights all-gathered
            res["allreduce_bytes_per_step"] = 0
            res["reduce_scatter_bytes_per_step"] = 4 * model.nparams
            res["all_gather_bytes_per_step"] = 2 * model.nparams

    # ---------------- profiled pass: per-launch events for the kernel split ----
    if profile:
        lib().rbk_ctx_profile(mctx, 1)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p_start.record(stream)
        for _ in range(steps):
            step()
        p_end.record(stream)
        torch.cuda.synchronize()
        prof_ms_step = p_start.elapsed_time(p_end) / steps
        cat_ms = (ctypes.c_double * 9)(); cat_w = (ctypes.c_double * 9)(); cat_n = (ctypes.c_int * 9)()
        lib().rbk_ctx_profile_read(mctx, cat_ms, cat_w, cat_n, 9)
        r_ms = (ctypes.c_double * 3)(); r_w = (ctypes.c_double * 3)(); r_n = (ctypes.c_int * 3)()
        lib().rbk_ctx_profile_read_gemm(mctx, r_ms, r_w, r_n)
        lib().rbk_ctx_profile(mctx, 0)
        res["kernels"] = {CAT_NAMES[c]: {"ms_per_step": cat_ms[c] / steps, "launches_per_step": cat_n[c] / steps,
                                         "share": cat_ms[c] / max(sum(cat_ms), 1e-9)} for c in range(9) if cat_n[c]}
        gemm_tflops = cat_w[0] / (cat_ms[0] * 1e-3) / 1e12 if cat_ms[0] > 0 else 0.0
        by_role = {}
        for i, role in enumerate(("fwd", "dgrad", "wgrad")):
            if r_n[i]:
                a = r_w[i] / (r_ms[i] * 1e-3) / 1e12
                by_role[role] = {"flops_per_step": r_w[i] / steps, "ms_per_step": r_ms[i] / steps,
                                 "launches_per_step": r_n[i] / steps, "achieved": a, "frac": a / tc_sustained}
        res["roofline"] = {
            "bound": "tensor", "kernel": "gemm_pair_kernel / gemm_kernel (tcgen05, all GEMMs of the step)",
            "achieved": gemm_tflops, "peak": tc_sustained, "unit": "TFLOP/s", "frac": gemm_tflops / tc_sustained,
            "traffic": GEMM_TRAFFIC_PER_LAUNCH if name == "gpt2-small" else None,
            "traffic_unit": "DRAM bytes per GEMM launch (ncu, each step shape captured alone, launch-weighted)",
            "peak_source": f"{peak_kind} bf16_tflops_sustained (FP16 and BF16 share the dense tensor rate)",
            "by_role": by_role,
            "gemm_flops_per_launch": cat_w[0] / max(cat_n[0], 1),
            "gemm_ms_per_launch": cat_ms[0] / max(cat_n[0], 1),
            "measured": "CUDA events around every GEMM launch in a second pass of the same steps",
            "profiled_pass_ms_per_step": prof_ms_step}

    # ---------------- end-to-end through the public API with host buffers ----
    if e2e:
        h_tok = torch.empty((B, S), dtype=torch.int32, pin_memory=True)
        h_tgt = torch.empty((B, S), dtype=torch.int32, pin_memory=True)
        h_tok.copy_(tokens.cpu()); h_tgt.copy_(targets.cpu())
        d_tok = torch.empty_like(tokens); d_tgt = torch.empty_like(targets)
        h_loss = torch.empty(1, dtype=torch.float32, pin_memory=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for _ in range(steps):
            d_tok.copy_(h_tok, non_blocking=True)
            d_tgt.copy_(h_tgt, non_blocking=True)
            loss = model.forward(d_tok, d_tgt, B, S)
            backward(d_tok, d_tgt)
            update()
            h_loss.copy_(loss.view(1), non_blocking=True)
            torch.cuda.current_stream().synchronize()
            _ = float(h_loss[0])
        e2e_s = time.perf_counter() - w0
        if world > 1:
            t = torch.tensor([e2e_s], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t[0])
        res["e2e"] = {"value": world * ntok * steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 2 * ntok * 4,
                      "d2h_bytes_per_step": 4}
    if dp_check and world > 1 and not lora:
        res["dp_check"] = check_dp(model, tokens, targets, B, S, world, dist, torch)
    res["loss_scale"] = model.loss_scale
    res["skipped_steps"] = model.scaler().overflow_steps
    if lora:
        res["lora"] = {"rank": lora["rank"], "alpha": lora["alpha"], "targets": "q,v",
                       "inf_injection": f"1 in {wl['inject_stride']} dlogits elements every {wl['inject_every']}th step"}
    model.close()
    del tokens, targets
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="rbk", choices=["rbk", "reference"])
    ap.add_argument("--workload", default="gpt2-small", choices=sorted(WORKLOADS))
    ap.add_argument("--no-ckpt", action="store_true", help="disable activation checkpointing")
    ap.add_argument("--no-micro", action="store_true", help="skip the HBM-bound kernel microbench")
    ap.add_argument("--no-tokenizer", action="store_true", help="skip the GPU BPE tokenizer bench (N = 1 only)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-ref-ops", action="store_true", help="skip timing the reference's own CPU ops")
    ap.add_argument("--no-1p3b", action="store_true", help="skip the second (1.3B) workload pass")
    ap.add_argument("--steps-1p3b", type=int, default=5)
    ap.add_argument("--bucket-mb", type=float, default=25.0)
    ap.add_argument("--dp-shard", type=int, default=int(os.environ.get("RBK_DP_SHARD", "1")),
                    help="1 (default): sharded optimizer under data parallelism (reduce-scatter, the tail on each "
                         "rank's slices, FP16 all-gather); 0: all-reduce and the whole tail on every rank")
    ap.add_argument("--kernel", default=None,
                    help="loop one kernel instead of the training step (gemm_* of gemm_shapes(), ln_bwd, xent, "
                         "attn_fwd, attn_bwd, adam_tail, bpe_encode, bpe_encode_256, bpe_decode)")
    args = ap.parse_args()
    if args.kernel:
        import torch
        from rbk import ops
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        return kernel_loop(args.kernel, args.steps, torch, ops)
    assert args.warmup >= 3 or args.impl == "reference" or os.environ.get("RBK_BENCH_ALLOW_FEW_WARMUP"), \
        "at least 3 warm-up steps"
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    from rbk import ops

    hbm_peak, _, _, _ = peaks()
    wl = WORKLOADS[args.workload]
    head = run_workload(args.workload, args, world, rank, local, dist, torch, args.steps, args.warmup,
                        dp_check=True)
    others = {}
    if args.workload == "gpt2-small" and not args.no_1p3b:
        # the 1.3B decoder of the same step, a short pass (its scaling curve rides on every --gpus N run)
        others["1.3b"] = run_workload("1.3b", args, world, rank, local, dist, torch, args.steps_1p3b, 3,
                                      e2e=False)
    extra = {}
    if rank == 0 and not args.no_micro:
        try:
            extra["microbench"] = microbench(ops, torch, hbm_peak)
        except Exception as exc:   # report, never hide
            extra["microbench"] = {"error": repr(exc)}
    if rank == 0 and world == 1 and not args.no_tokenizer:
        try:
            extra["tokenizer"] = tokenizer_bench(torch, hbm_peak, cpu=not args.no_cpu)
        except Exception as exc:   # report, never hide
            extra["tokenizer"] = {"error": repr(exc)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, dt, cores = cpu_sample(args.workload)
        seq = CPU_SEQ[args.workload]
        cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"oracle fwd+bwd+AdamW{' (LoRA adapters)' if wl.get('lora') else ''} of the same model "
                         f"over 1 x {seq} tokens ({dt:.1f} s, {cores} threads)"}
        if not args.no_ref_ops and args.workload != "tiny":
            cpu["reference_ops"] = reference_ops()
    if world > 1:
        dist.barrier()
    if rank == 0:
        out = {
            "metric": METRIC, "value": head["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic (uniform random tokens, N(0,0.02) weights)",
            "config": {"workload": wl["name"], "global_batch": head["global_batch"], "seq_len": head["seq_len"],
                       "parallelism": f"dp{world}", "activation_checkpointing": head["activation_checkpointing"],
                       "loss_scale_init": 65536,
                       "l2": "no flush: weights/activations/logits exceed 126 MB L2",
                       "value_scope": "whole job: tokens/s summed over all N GPUs; tokens_per_s_per_gpu = value / N"},
            "tokens_per_s_per_gpu": head["tokens_per_s_per_gpu"],
            "backward_ms_per_step": head["backward_ms_per_step"],
            "train_tflops_per_gpu": head["train_tflops_per_gpu"],
            "gemm_flops_per_step": head["gemm_flops_per_step"],
            "roofline": head.get("roofline"),
            "kernels": head.get("kernels"),
            "e2e": head.get("e2e"),
            "gpu_launches": head["gpu_launches"],
            "clocks": head["clocks"],
            "cpu_baseline": cpu,
            "loss_scale": head["loss_scale"],
            "skipped_steps": head["skipped_steps"],
        }
        for k in ("dp_check", "allreduce_bytes_per_step", "reduce_scatter_bytes_per_step", "all_gather_bytes_per_step",
                  "sharded_optimizer", "lora"):
            if k in head:
                out[k] = head[k]
        if others:
            out["workloads"] = others
        out.update(extra)
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
