"""Benchmark of the WKV-7 + ROSA hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the hot path over one batch of synthetic input.  The
headline workload is the isolated WKV-7 scan op of benchmark config 2
(B=8, T=2048, H=16, N=40, fp32, zero initial state, seeded N(0,1) inputs):
each rank scans its own batch (weak scaling, no collective on the data path;
NCCL only for the start/stop barrier and the max-over-ranks time).

* ``value``   tokens/s over all ranks, inputs resident in HBM (device-timed).
* ``e2e``     the same metric through the public API (``cuda_ops.rwkv7_cuda``)
              with pinned HOST buffers: every step copies the inputs to the
              device and y + final state back; the copies of neighbouring
              steps overlap the scan on their own streams (double-buffered).
* ``roofline``  the scan's algorithmic bytes (6 inputs + y per (b,t,h):
              7*N*4 B; plus the final state N*N*4 per (b,h)) over the measured
              time of one step, against the measured HBM copy bandwidth.  At
              this shape (B*H = 128 chains, one 86 %-full wave of CTAs) AUTO runs
              the chunked tensor-core scan: one launch of
              wkv7_chunk_tc_kernel<40> per step.
* ``cpu_baseline``  the C restatement of the reference recurrence
              (oracle/scans_ref.c, OpenMP over (b,h)) on this host's cores;
              ``cpu_baseline_model`` the whole 0.1B model through the numpy port
              of the reference's CPU forward/step on bounded samples (N = 1).
* ``sharded``  benchmark configs 3 (the 0.1B model's B2 x T2048 prefill,
              fp32 and bf16 weights, one replica per rank: B = 2 does not
              shard further), 4 (256 sequences x 1024 generated tokens, top-k
              32, through Engine.generate, 256 / N sequences per rank) and 5 (8
              sequences of 8192 tokens per GPU, bf16 weights), each timed as the
              max over ranks: prefill and decode tokens/s at N GPUs.  Their
              headline figures are repeated as short top-level keys
              (``prefill_c3_tokens_per_s``, ``decode_c4_tokens_per_s``, ...; all
              totals over the N GPUs, with ``*_per_gpu`` and roofline fractions)
              so every N of a scaling run carries them; the config-4 HBM fraction
              counts decode steps only (the prompt prefill's time is taken out).
* ``extra``   rank 0's secondary kernel and model timings (sequential and
              chunked scans, decode step, ROSA, backward, 0.1B prefill/decode).

``--impl reference`` times the reference algorithm's CPU implementation
(the same C port; the reference itself is PyTorch CPU code that cannot be
shipped to the GPU box) on rank 0 and prints its own line, with the whole
model's CPU port timed on bounded samples of configs 3 and 4 under the same
top-level keys.  Both ports are faster than the reference's PyTorch CPU
fallback (a Python loop of einsums per token), so they are stronger baselines.

``--only headline`` runs just the config-2 steps (the command the profiles'
ncu captures use); ``--only scans`` every scan algorithm once on config 2;
``--only model`` just one rank's config-3 prefill and
config-4 decode step timings (fp32 and bf16 weights); ``--only prefill`` /
``--only decode`` just the bf16-weight config-3 prefill / config-4 decode step;
``--only c5`` one rank's config-5 prefill (8 sequences of 8192 tokens).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B, T, H, N = 8, 2048, 16, 40
TOKENS = B * T
ALGO_BYTES = B * T * H * 7 * N * 4 + B * H * N * N * 4
METRIC = "wkv7_scan_prefill_tokens_per_s"
UNIT = "tokens/s"
WORKLOAD = "config2_wkv7_scan_op_B8_T2048_H16_N40_fp32"
LAUNCHES_PER_STEP = 1  # the chunked tensor-core scan (AUTO at B*H = 128)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--only", choices=["all", "headline", "scans", "model", "prefill", "decode", "c5"],
                   default="all")
    return p.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_peak():
    """Measured bf16 dense TFLOP/s (sustained: the prefill is a long step)."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))
    return 1400.0


def profiled_traffic():
    """DRAM bytes of one headline step from the committed ncu summary of the
    chunked tensor-core scan on the config-2 workload."""
    f = ROOT / "profiles" / "wkv7_chunk_tc_config2.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_step:"):
            return float(line.split(":", 1)[1])
    return None


def cpu_oracle_run(n_batch, seconds, threads=None):
    from oracle import cref
    from yufmusicgen_b200.workloads import wkv_op_inputs

    ins = wkv_op_inputs(n_batch, T, H, N, seed=0)
    args = [ins[k] for k in "rwkvab"]
    cref.wkv7_scan(*args, n_threads=threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        cref.wkv7_scan(*args, n_threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n_batch * T * reps / el, reps, el


def cpu_model_baseline():
    """The whole model on the host cores: the numpy port of YufMusicGen.forward /
    .step (oracle/model.py, the reference's use_rosa_scan=False CPU path) on
    bounded samples of benchmark configs 3 (prefill) and 4 (decode)."""
    from oracle.model import OracleModel
    from yufmusicgen_b200 import config as C
    from yufmusicgen_b200.weights import init_weights
    from yufmusicgen_b200.workloads import zipf_ids

    try:
        from threadpoolctl import threadpool_info
        threads = max((d.get("num_threads", 1) for d in threadpool_info()), default=1)
    except Exception:  # pragma: no cover - threadpoolctl is optional
        threads = os.cpu_count()
    cfg = C.ModelConfig(**C.BASE_0P1B)
    om = OracleModel(cfg, init_weights(cfg, 1, "baseline"))
    ids = zipf_ids(1, 512, seed=1, vocab=cfg.vocab_size)
    t0 = time.perf_counter()
    om.forward(ids)
    pf = 512 / (time.perf_counter() - t0)
    seqs, steps = 32, 8
    logits, st = om.forward(zipf_ids(seqs, C4_PROMPT, seed=4, vocab=cfg.vocab_size))
    tok = np.argmax(logits[:, -1], axis=-1)
    t0 = time.perf_counter()
    for _ in range(steps):
        last, st = om.step(tok, st)
        tok = np.argmax(last, axis=-1)
    dec = seqs * steps / (time.perf_counter() - t0)
    return {"prefill_c3_tokens_per_s": pf, "decode_c4_tokens_per_s": dec, "unit": "tokens/s",
            "cores": threads, "kind": "port",
            "sample": "config-3 model (fp32): prefill of 1 x 512 tokens; greedy decode of 32 of "
                      "config 4's sequences x 8 steps after their 64-token prompts; numpy port "
                      "of the reference's CPU forward/step"}


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return
    from oracle import cref

    threads = cref.threads_default()
    sample_b = 2
    from yufmusicgen_b200.workloads import wkv_op_inputs

    ins = wkv_op_inputs(sample_b, T, H, N, seed=0)
    a = [ins[k] for k in "rwkvab"]
    for _ in range(args.warmup):
        cref.wkv7_scan(*a, n_threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cref.wkv7_scan(*a, n_threads=threads)
    el = time.perf_counter() - t0
    value = sample_b * T * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample": f"B{sample_b} of B{B} per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample_b} of {B} sequences x T{T} x H{H} per step; C port of "
                                   "RWKV7TimeMix._torch_recurrence, OpenMP over (b,h)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    # the whole model on the same host cores, bounded samples of configs 3 and 4,
    # under the keys of our arm's line (totals: one host serves every N)
    mb = cpu_model_baseline()
    line.update({"prefill_c3_tokens_per_s": mb["prefill_c3_tokens_per_s"],
                 "prefill_c3_fp32_tokens_per_s": mb["prefill_c3_tokens_per_s"],
                 "decode_c4_tokens_per_s": mb["decode_c4_tokens_per_s"],
                 "decode_c4_fp32_tokens_per_s": mb["decode_c4_tokens_per_s"],
                 "cpu_baseline_model": mb})
    print(json.dumps(line), flush=True)


def _time(fn, n, dev, stream, warm=3):
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / n


SCAN_ALGOS = (("sequential", "ALGO_SEQUENTIAL"), ("chunked16", "ALGO_CHUNKED"),
              ("time_parallel", "ALGO_PARALLEL"), ("rows", "ALGO_ROWS"), ("chunked_tc", "ALGO_CHUNKED_TC"))


def measure_scans(dev, stream, args):
    """Every WKV-7 scan algorithm on the headline workload (config 2), each
    called explicitly (``--only scans``; the profiles' captures of the kernels
    that AUTO does not pick at this shape use it)."""
    import torch

    from yufmusicgen_b200 import cuda_ops
    from yufmusicgen_b200.workloads import wkv_op_inputs

    out = {}
    n = max(5, min(args.steps, 50))
    ins = wkv_op_inputs(B, T, H, N, seed=0)
    d = {k: torch.from_numpy(ins[k]).to(dev) for k in "rwkvab"}
    y = torch.empty_like(d["r"])
    s = torch.empty(B, H, N, N, device=dev)
    for name, algo in SCAN_ALGOS:
        a = getattr(cuda_ops, algo)
        ms = _time(lambda: cuda_ops.wkv7_forward(*(d[k] for k in "rwkvab"), None, out=y, state_out=s,
                                                 algo=a), n, dev, stream)
        out[f"wkv7_{name}_config2"] = {"ms": ms, "GBps": ALGO_BYTES / ms / 1e6}
    del d, y, s
    return out


def measure_extras(dev, stream, args):
    """Secondary kernels of the hot path, timed on rank 0 (not the headline)."""
    import torch

    from yufmusicgen_b200 import cuda_ops, rosa_cuda
    from yufmusicgen_b200.workloads import rosa_op_inputs, wkv_op_inputs

    peak, _ = peaks()
    n = max(5, min(args.steps, 50))
    # every scan algorithm on the headline workload, for comparison
    out = measure_scans(dev, stream, args)
    # batched decode step: config-4 state shape (256 seqs x 16 heads x N40), T = 1
    Bd = 256
    di = wkv_op_inputs(Bd, 1, H, N, seed=1, with_state=True)
    dd = {k: torch.from_numpy(di[k]).to(dev) for k in "rwkvab"}
    yd = torch.empty_like(dd["r"])
    # eight in-place states (8 x 26 MB > L2), one CUDA graph of eight steps so the
    # number is the kernel's, not the Python call's
    sts = [torch.from_numpy(di["s0"]).to(dev) for _ in range(8)]

    def dec_all():
        for st in sts:
            cuda_ops.wkv7_forward(*(dd[k] for k in "rwkvab"), st, out=yd, state_out=st,
                                  algo=cuda_ops.ALGO_SEQUENTIAL)

    def floor_all():  # an in-place float update of the same states: the streaming floor
        for st in sts:
            st.mul_(1.0)

    def graph_ms(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        t = _time(g.replay, n, dev, stream) / len(sts)
        del g
        return t

    ms = graph_ms(dec_all)
    ms_floor = graph_ms(floor_all)
    dbytes = 2 * Bd * H * N * N * 4 + 7 * Bd * H * N * 4
    out["wkv7_decode_step_B256_H16_N40"] = {"ms": ms, "GBps": dbytes / ms / 1e6,
                                            "frac_of_hbm": dbytes / ms / 1e6 / peak,
                                            "inplace_update_floor_ms": ms_floor,
                                            "frac_of_inplace_floor": ms_floor / ms,
                                            "bytes": dbytes}
    del sts
    # ROSA scan at the 0.1B model's shape (B2, T2048, R128), gated
    ri = rosa_op_inputs(2, T, 128, seed=2)
    keys = ("cand", "write", "read_gate", "decay", "direction", "m0")
    rd = [torch.from_numpy(ri[k]).to(dev) for k in keys]
    ro = torch.empty_like(rd[0])
    mo = torch.empty_like(rd[5])
    ms = _time(lambda: rosa_cuda.rosa_scan(*rd, gated=True, out=ro, memory_out=mo), n, dev, stream)
    rbytes = 4 * 2 * T * 128 * 4
    out["rosa_scan_B2_T2048_R128"] = {"ms": ms, "GBps": rbytes / ms / 1e6,
                                      "tokens_per_s": 2 * T / (ms * 1e-3)}
    del rd, ro, mo
    # training backward at the config-2 and config-3 ROSA shapes (after the compat forward)
    ins = wkv_op_inputs(B, T, H, N, seed=0)
    d = [torch.from_numpy(ins[k]).to(dev) for k in "rwkvab"]
    y, states, sa = cuda_ops.wkv7_forward_compat(*d)
    dy = torch.randn_like(y)
    grads = [torch.empty_like(y) for _ in range(6)]
    ms = _time(lambda: cuda_ops.wkv7_backward(*d, dy, states, sa, grads), n, dev, stream)
    out["wkv7_backward_config2"] = {"ms": ms, "tokens_per_s": B * T / (ms * 1e-3)}
    del d, y, states, sa, dy, grads
    ri = rosa_op_inputs(2, T, 128, seed=2, with_state=True)
    rd = [torch.from_numpy(ri[k]).to(dev) for k in keys]
    _, m_out, saved, mem_saved = rosa_cuda.rosa_forward_compat(*rd)
    dq = torch.randn_like(rd[0])
    ms = _time(lambda: rosa_cuda.rosa_backward(*saved, mem_saved, rd[4], m_out, dq), n, dev, stream)
    out["rosa_backward_B2_T2048_R128"] = {"ms": ms, "tokens_per_s": 2 * T / (ms * 1e-3)}
    del rd, saved, mem_saved, dq
    out.update(measure_model(dev, stream))
    return out


C4_SEQS, C4_PROMPT, C4_STEPS = 256, 64, 1024
C5_SEQS_PER_GPU, C5_T = 8, 8192


def model_bytes_per_step(cfg, wsz):
    """Bytes a decode step must move for one model: every weight once (the tied
    embedding as the LM head) and, per sequence, the recurrent state in and out
    (per layer prev [d], S [H,N,N], m [R]) plus its logits row."""
    d, lr, R, V = cfg.d_model, cfg.low_rank, cfg.rosa_size, cfg.vocab_size
    per_layer = 4 * d * d + 6 * d * lr + 3 * R * d + R * d + 12 * d * d
    weights = (cfg.n_layers * per_layer + V * d) * wsz
    state = cfg.n_layers * 2 * 4 * (d + cfg.n_heads * cfg.head_size ** 2 + R) + 4 * V
    return weights, state


C3_FLOP_PER_TOKEN = 225e6  # about 2 x non-embedding linear parameters + the LM head


def measure_sharded(dev, rank, world, barrier, max_over_ranks):
    """Benchmark configs 3, 4 and 5 on every rank, each timed as the max over
    ranks of each rank's CUDA-event time (no collective on the data path).

    * config 3: the 0.1B model's prefill of B2 x T2048 (the ids of the
      reference fixture tests/golden/model_c3_full.npz), fp32 and bf16 weights;
      one replica per rank (B = 2 sequences do not shard over more GPUs).
    * config 4: 256 sequences (256 / world per GPU), 64-token prompts
      (Zipf(1.1) after a byte prefix), 1024 tokens generated per sequence with
      temperature 1.0 and top-k 32 under Philox seed 2024 through
      ``Engine.generate`` (yuf_generate: on-device sampling, CUDA-graph decode
      steps).  The time covers the prefill and all 1024 steps; the prompt
      prefill alone is timed too, so the decode steps' HBM fraction excludes it.
    * config 5: 8 of the 64 sequences of T = 8192 per GPU through the 24-layer
      d1024 model (bf16 weights, fp32 state): prefill tokens/s.
    """
    import torch

    from yufmusicgen_b200 import config as C
    from yufmusicgen_b200.engine import Engine
    from yufmusicgen_b200.weights import init_weights
    from yufmusicgen_b200.workloads import zipf_ids

    peak, _ = peaks()
    res = {}
    side = torch.cuda.Stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, reps, stream):
        fn()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / reps)

    cfg = C.ModelConfig(**C.BASE_0P1B)
    w = init_weights(cfg, 1, "baseline")
    # config 3: B2 x T2048 prefill, a replica per rank
    ids3 = torch.as_tensor(zipf_ids(2, 2048, seed=1, vocab=cfg.vocab_size), dtype=torch.int32, device=dev)
    for prec in ("bf16", "fp32"):
        eng = Engine(cfg, w, precision=prec, device=dev.index, n_slots=2)
        last = torch.empty(2, cfg.vocab_size, device=dev)

        def pf3():
            eng.reset_state(0, 2)
            eng.prefill(ids3, slot0=0, out_last=last)

        ms = timed(pf3, 5, torch.cuda.current_stream(dev))
        tok = world * 2 * 2048
        tflops = C3_FLOP_PER_TOKEN * 2 * 2048 / (ms * 1e-3) / 1e12
        res[f"prefill_c3_{prec}"] = {"ms": ms, "tokens_per_s": tok / (ms * 1e-3), "sequences": 2 * world,
                                     "seq_len": 2048, "replicas": world, "TFLOPs_per_gpu": tflops,
                                     "tensor_frac_per_gpu": tflops / bf16_peak()}
        eng.close()
        del eng
    per = C4_SEQS // world
    prompt = torch.as_tensor(zipf_ids(C4_SEQS, C4_PROMPT, seed=4, vocab=cfg.vocab_size)[rank * per:(rank + 1) * per],
                             dtype=torch.int32, device=dev)
    gen = dict(temperature=1.0, top_k=32, seed=2024, seq0=rank * per)
    for prec in ("bf16", "fp32"):
        with torch.cuda.stream(side):
            eng = Engine(cfg, w, precision=prec, device=dev.index, n_slots=per)
            eng.set_decode_graphs(True)
            toks = torch.empty(per, C4_STEPS, dtype=torch.int32, device=dev)
            lens = torch.empty(per, dtype=torch.int32, device=dev)
            last = torch.empty(per, cfg.vocab_size, device=dev)

            def prompt_prefill():
                eng.reset_state(0, per)
                eng.prefill(prompt, slot0=0, out_last=last)

            pre_ms = timed(prompt_prefill, 3, side)
            eng.generate(prompt, 8, out_tokens=toks[:, :8].contiguous(), out_lengths=lens, **gen)
            ms = timed(lambda: (eng.reset_state(0, per),
                                eng.generate(prompt, C4_STEPS, out_tokens=toks, out_lengths=lens, **gen)),
                       1, side)
            wbytes, sbytes = model_bytes_per_step(cfg, 2 if prec == "bf16" else 4)
            step_ms = max(ms - pre_ms, 1e-6) / C4_STEPS  # decode steps only
            step_bytes = wbytes + per * sbytes
            res[f"generate_c4_{prec}"] = {
                "ms": ms, "prompt_prefill_ms": pre_ms, "decode_ms_per_step": step_ms,
                "tokens_per_s": C4_SEQS * C4_STEPS / (ms * 1e-3),
                "decode_tokens_per_s": C4_SEQS / (step_ms * 1e-3),
                "sequences": C4_SEQS, "sequences_per_gpu": per, "prompt": C4_PROMPT, "steps": C4_STEPS,
                "sampler": "temperature 1.0, top-k 32, Philox4x32-10 seed 2024 on device",
                "step_bytes_per_gpu": step_bytes,
                "hbm_frac_per_gpu": step_bytes / (step_ms * 1e-3) / 1e9 / peak}
            eng.close()
            del eng
    del w
    # config 5: this rank's 8 of the 64 sequences
    ms = measure_c5(dev, 2, rank, timed)
    tokens = world * C5_SEQS_PER_GPU * C5_T
    flop = 915e6 * tokens  # about 2 x linear parameters + LM head per token
    tflops = flop / world / (ms * 1e-3) / 1e12
    res["prefill_c5_bf16"] = {"ms": ms, "tokens_per_s": tokens / (ms * 1e-3),
                              "sequences": world * C5_SEQS_PER_GPU, "seq_len": C5_T,
                              "TFLOPs_per_gpu": tflops,
                              "tensor_frac_per_gpu": tflops / bf16_peak()}
    return res


def measure_c5(dev, reps, rank=0, timed=None):
    """Config 5 on one rank: 8 sequences of T = 8192 through the 24-layer d1024
    model (bf16 weights, fp32 state); ms per prefill (max over ranks when
    `timed` is the sharded timer)."""
    import torch

    from yufmusicgen_b200 import config as C
    from yufmusicgen_b200.engine import Engine
    from yufmusicgen_b200.weights import init_weights
    from yufmusicgen_b200.workloads import zipf_ids

    cfg = C.ModelConfig(**C.LONG_1K)
    w = init_weights(cfg, 2, "baseline")
    ids = torch.as_tensor(zipf_ids(C5_SEQS_PER_GPU, C5_T, seed=100 + rank, vocab=cfg.vocab_size),
                          dtype=torch.int32, device=dev)
    eng = Engine(cfg, w, precision="bf16", device=dev.index, n_slots=C5_SEQS_PER_GPU)
    del w
    last = torch.empty(C5_SEQS_PER_GPU, cfg.vocab_size, device=dev)

    def pf():
        eng.reset_state(0, C5_SEQS_PER_GPU)
        eng.prefill(ids, slot0=0, out_last=last)

    stream = torch.cuda.current_stream(dev)
    if timed is None:
        ms = _time(pf, reps, dev, stream, warm=1)
        out = {"ms": ms, "tokens_per_s": C5_SEQS_PER_GPU * C5_T / (ms * 1e-3)}
    else:
        out = timed(pf, reps, stream)
    eng.close()
    del eng
    return out


def headline_keys(sh, world):
    """Short top-level keys of the model-level figures (totals over the N GPUs)."""
    c3, c3f = sh["prefill_c3_bf16"], sh["prefill_c3_fp32"]
    c4, c4f = sh["generate_c4_bf16"], sh["generate_c4_fp32"]
    c5 = sh["prefill_c5_bf16"]
    return {
        "prefill_c3_tokens_per_s": c3["tokens_per_s"],
        "prefill_c3_tokens_per_s_per_gpu": c3["tokens_per_s"] / world,
        "prefill_c3_tensor_frac": c3["tensor_frac_per_gpu"],
        "prefill_c3_fp32_tokens_per_s": c3f["tokens_per_s"],
        "decode_c4_tokens_per_s": c4["decode_tokens_per_s"],
        "decode_c4_tokens_per_s_per_gpu": c4["decode_tokens_per_s"] / world,
        "decode_c4_hbm_frac": c4["hbm_frac_per_gpu"],
        "decode_c4_ms_per_step": c4["decode_ms_per_step"],
        "decode_c4_fp32_tokens_per_s": c4f["decode_tokens_per_s"],
        "generate_c4_tokens_per_s": c4["tokens_per_s"],
        "prefill_c5_tokens_per_s": c5["tokens_per_s"],
        "prefill_c5_tensor_frac": c5["tensor_frac_per_gpu"],
    }


def measure_model(dev, stream, parts=("prefill", "decode"), precisions=("fp32", "bf16")):
    """The 0.1B model (benchmark config 3/4 shapes) through the engine:
    prefill tokens/s (B2 x T2048) in fp32 and bf16-weight mode, and batched
    greedy decode tokens/s (256 sequences, 64-token prompts, config 4's batch)."""
    import torch

    from yufmusicgen_b200 import config as C
    from yufmusicgen_b200.engine import Engine
    from yufmusicgen_b200.sampler import sample
    from yufmusicgen_b200.weights import init_weights
    from yufmusicgen_b200.workloads import zipf_ids

    cfg = C.ModelConfig(**C.BASE_0P1B)
    w = init_weights(cfg, 1, "baseline")
    res = {}
    ids = torch.as_tensor(zipf_ids(2, 2048, seed=1, vocab=cfg.vocab_size), dtype=torch.int32, device=dev)
    for prec in (precisions if "prefill" in parts else ()):
        eng = Engine(cfg, w, precision=prec, device=dev.index, n_slots=2)
        last = torch.empty(2, cfg.vocab_size, device=dev)

        def pf():
            eng.reset_state(0, 2)
            eng.prefill(ids, slot0=0, out_last=last)

        ms = _time(pf, 3, dev, stream, warm=1)
        res[f"prefill_0p1b_B2_T2048_{prec}"] = {"ms": ms, "tokens_per_s": 2 * 2048 / (ms * 1e-3)}
        eng.close()
        del eng
    # batched decode, config 4 shape: 256 sequences, 64-token byte prompts
    Bd, steps = 256, 32
    side = torch.cuda.Stream(dev)
    for prec in (precisions if "decode" in parts else ()):
      with torch.cuda.stream(side):
        eng = Engine(cfg, w, precision=prec, device=dev.index, n_slots=Bd)
        eng.set_decode_graphs(True)
        prompt = torch.as_tensor(zipf_ids(Bd, 64, seed=4, vocab=cfg.vocab_size), dtype=torch.int32,
                                 device=dev)
        logits = eng.prefill(prompt)
        tok = torch.argmax(logits, dim=-1).to(torch.int32)
        out_l = torch.empty(Bd, cfg.vocab_size, device=dev)

        step_no = [0]

        def dec():
            eng.step(tok, out=out_l)  # same buffers every step -> one captured graph
            sample(out_l, seed=1234, step=step_no[0], temperature=1.0, top_k=32, out=tok)
            step_no[0] += 1

        ms = _time(dec, steps, dev, side, warm=2)
        res[f"decode_0p1b_B256_{prec}"] = {"ms_per_step": ms, "tokens_per_s": Bd / (ms * 1e-3),
                                           "sampler": "top-k 32, T=1.0, Philox4x32-10 on device",
                                           "cuda_graph": True}
        eng.close()
        del eng
    return res


def run_ours(args):
    import torch

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = world > 1
    if dist:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=dev)
    from yufmusicgen_b200 import cuda_ops
    from yufmusicgen_b200.telemetry import ClockSampler
    from yufmusicgen_b200.workloads import wkv_op_inputs

    def barrier():
        if dist:
            torch.distributed.barrier()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    ins = wkv_op_inputs(B, T, H, N, seed=rank)
    # the six inputs in one pinned host buffer (one copy per step), allocated by
    # this rank's process after set_device so its pages are touched by its thread
    host_all = torch.empty(6, B, T, H, N).pin_memory()
    for i, k in enumerate("rwkvab"):
        host_all[i].copy_(torch.from_numpy(ins[k]))
    host = {k: host_all[i] for i, k in enumerate("rwkvab")}
    d = {k: host[k].to(dev) for k in "rwkvab"}
    y = torch.empty_like(d["r"])
    s = torch.empty(B, H, N, N, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        cuda_ops.wkv7_forward(d["r"], d["w"], d["k"], d["v"], d["a"], d["b"], None, out=y, state_out=s)

    if args.only == "c5":
        print(json.dumps({"only": "c5", "c5": measure_c5(dev, 1)}), flush=True)
        return
    if args.only == "scans":
        print(json.dumps({"only": "scans", "scans": measure_scans(dev, stream, args)}), flush=True)
        return
    if args.only in ("model", "prefill", "decode"):
        parts = ("prefill", "decode") if args.only == "model" else (args.only,)
        precs = ("fp32", "bf16") if args.only == "model" else ("bf16",)
        print(json.dumps({"only": args.only, "model": measure_model(dev, stream, parts, precs)}), flush=True)
        return
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms)
    value = world * TOKENS / (ms_max * 1e-3)
    if args.only == "headline":
        if rank == 0:
            print(json.dumps({"only": "headline", "ms_per_step": ms_max, "value": value}), flush=True)
        if dist:
            torch.distributed.destroy_process_group()
        return

    # End to end through the public API with pinned host buffers: every step copies its six
    # inputs host->device and its outputs (y, final state) device->host.  The copies run on
    # their own streams with two device buffer sets, so step i's input copy, step i-1's scan
    # and step i-2's output copy overlap (PCIe is full duplex); the timed region ends when the
    # last output copy has landed.
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dall = [torch.empty(6, B, T, H, N, device=dev) for _ in range(2)]
    dbuf = [{k: dall[j][i] for i, k in enumerate("rwkvab")} for j in range(2)]
    y_h = [torch.empty(B, T, H, N).pin_memory() for _ in range(2)]
    s_h = [torch.empty(B, H, N, N).pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer set i landed
    ev_comp = [torch.cuda.Event() for _ in range(2)]  # the scan that read set i is done
    ev_out = [torch.cuda.Event() for _ in range(2)]   # outputs of set i copied to the host
    step_no = [0]

    def e2e_step():
        i = step_no[0] % 2
        step_no[0] += 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_comp[i])
            dall[i].copy_(host_all, non_blocking=True)
            ev_in[i].record(s_in)
        stream.wait_event(ev_in[i])
        stream.wait_event(ev_out[i])
        yy, ss = cuda_ops.rwkv7_cuda(*(dbuf[i][k] for k in "rwkvab"))
        ev_comp[i].record(stream)
        yy.record_stream(s_out)
        ss.record_stream(s_out)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[i])
            y_h[i].copy_(yy, non_blocking=True)
            s_h[i].copy_(ss, non_blocking=True)
            ev_out[i].record(s_out)

    e2e_steps = max(2, min(args.steps, 50))
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    stream.wait_event(ev_out[0])
    stream.wait_event(ev_out[1])
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    h2d = host_all.numel() * 4
    d2h = (y_h[0].numel() + s_h[0].numel()) * 4
    # the input copy alone, all ranks at once: the host -> device bandwidth each
    # rank gets (the e2e limiter: the scan takes a twentieth of the copy's time)
    torch.cuda.synchronize(dev)
    barrier()
    e0.record(s_in)
    for _ in range(5):
        dall[0].copy_(host_all, non_blocking=True)
    e1.record(s_in)
    torch.cuda.synchronize(dev)
    barrier()
    h2d_ms = max_over_ranks(e0.elapsed_time(e1) / 5)

    sharded = measure_sharded(dev, rank, world, barrier, max_over_ranks)
    extra = measure_extras(dev, stream, args) if rank == 0 else {}

    if rank == 0:
        peak, peak_kind = peaks()
        achieved = ALGO_BYTES / (ms * 1e-3) / 1e9
        traffic = profiled_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "per_gpu_batch": B, "seq_len": T, "heads": H,
                       "head_size": N, "parallelism": f"batch-sharded x{world}, no collectives",
                       "l2": "inputs larger than L2 (294 MB touched per step)"},
            "e2e": {"value": world * TOKENS / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "h2d_GBps_per_rank_alone": h2d / (h2d_ms * 1e-3) / 1e9,
                    "h2d_GBps_per_rank_in_e2e": h2d / (e2e_ms * 1e-3) / 1e9,
                    "limiter": "host->device copy of the inputs (one pinned buffer per rank, "
                               "all ranks at once); the scan overlaps it"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "wkv7 chunked tensor-core scan (AUTO at B*H = 128): "
                                   "wkv7_chunk_tc_kernel<40>",
                         "algorithmic_bytes_per_step": ALGO_BYTES},
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "clocks": clocks.summary(),
            **headline_keys(sharded, world),
            "sharded": sharded,
            "extra": extra,
        }
        if world == 1:
            v, reps, el = cpu_oracle_run(B, seconds=3.0)
            from oracle import cref

            line["cpu_baseline"] = {
                "value": v, "unit": UNIT, "cores": cref.threads_default(), "kind": "port",
                "sample": f"full config-2 workload x{reps} ({el:.1f} s); C port of the reference "
                          "recurrence, OpenMP over (b,h)",
                "note": "a stronger baseline than the reference's PyTorch CPU fallback (a Python "
                        "loop of einsums per token), which the port outruns 40-80x"}
            line["cpu_baseline_model"] = cpu_model_baseline()
        print(json.dumps(line), flush=True)
    if dist:
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
