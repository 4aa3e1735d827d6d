"""Generate the golden fixtures from the reference implementation itself.

Run in a container that holds the reference source tree (it is imported, not
copied):

    YUF_REFERENCE=/path/to/YufMusicGen python tests/golden/make_golden.py

Every fixture is produced by the reference's own PyTorch fp32 CPU code:

* ``RWKV7TimeMix._torch_recurrence``   (yufmusicgen/model.py:145-165)
* ``ROSAMemory._reference_recurrence`` (yufmusicgen/model.py:260-288)
* ``YufMusicGen.forward`` / ``.step``  (yufmusicgen/model.py:406-431) built with
  ``use_cuda_kernel=False, use_rosa_scan=False`` and loaded with the seeded
  weights of ``yufmusicgen_b200.weights.init_weights``.
* gradients of both recurrences by torch autograd through the reference's
  CPU code (``grads_cases.npz``), the oracle of the training backward ops.

``python tests/golden/make_golden.py dropin`` writes only the fixture of the
reference op wrapper's own padding (``yufmusicgen/cuda_ops.py`` ``_pad_inputs``:
T padded to a multiple of 16 with w_raw = -80 and zeros) with the CPU
recurrence's output for the unpadded inputs (``dropin_pad_cases.npz``);
``python tests/golden/make_golden.py grads`` writes only the gradient fixture,
``... greedy256`` only the 256-step greedy decode of the 0.1B model, ``... long``
only the benchmark-size prefills (config 3 in full, config-5 geometry), ``...
sampler`` only the reference's sampled-decode draws.

The fixtures are small ``.npz`` files; the GPU box never needs the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
REF = os.environ.get("YUF_REFERENCE")
if not REF:
    raise SystemExit("set YUF_REFERENCE to the reference source tree")
sys.path.insert(0, REF)
sys.dont_write_bytecode = True

import torch  # noqa: E402
from yufmusicgen.config import ModelConfig as RefConfig  # noqa: E402
from yufmusicgen.model import ROSAMemory, RWKV7TimeMix, YufMusicGen  # noqa: E402

from yufmusicgen_b200 import config as C  # noqa: E402
from yufmusicgen_b200.weights import init_weights  # noqa: E402
from yufmusicgen_b200.workloads import rosa_op_inputs, tiny_ids, wkv_op_inputs, zipf_ids  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def t(x):
    return torch.from_numpy(np.ascontiguousarray(x))


def wkv_cases():
    out = {}
    cases = [
        ("n40_state", 2, 37, 3, 40, 11, True),
        ("n32_zero", 1, 16, 2, 32, 12, False),
        ("n64_state", 2, 9, 2, 64, 13, True),
        ("n16_state", 3, 21, 2, 16, 14, True),
        ("n40_t1", 4, 1, 5, 40, 15, True),
    ]
    for name, B, T, H, N, seed, st in cases:
        ins = wkv_op_inputs(B, T, H, N, seed=seed, with_state=st)
        s0 = ins["s0"] if st else np.zeros((B, H, N, N), np.float32)
        y, sT = RWKV7TimeMix._torch_recurrence(
            t(ins["r"]), t(ins["w"]), t(ins["k"]), t(ins["v"]), t(ins["a"]), t(ins["b"]), t(s0)
        )
        for k in ("r", "w", "k", "v", "a", "b"):
            out[f"{name}.{k}"] = ins[k]
        out[f"{name}.s0"] = s0
        out[f"{name}.y"] = y.numpy()
        out[f"{name}.sT"] = sT.numpy()
    np.savez_compressed(HERE / "wkv7_cases.npz", **out)


def rosa_cases():
    out = {}
    cases = [
        ("r32_state", 2, 29, 32, 21, True),
        ("r128_zero", 2, 33, 128, 22, False),
        ("r256_state", 1, 17, 256, 23, True),
        ("r12_state", 3, 7, 12, 24, True),
        ("r128_t1", 5, 1, 128, 25, True),
    ]
    for name, B, T, R, seed, st in cases:
        ins = rosa_op_inputs(B, T, R, seed=seed, with_state=st)
        read, mT = ROSAMemory._reference_recurrence(
            t(ins["cand"]), t(ins["write"]), t(ins["read_gate"]), t(ins["decay"]),
            t(ins["direction"]), t(ins["m0"]),
        )
        for k, v in ins.items():
            out[f"{name}.{k}"] = v
        out[f"{name}.read"] = read.numpy()
        out[f"{name}.mT"] = mT.numpy()
    np.savez_compressed(HERE / "rosa_cases.npz", **out)


def grad_cases():
    """dL/d(inputs) for L = sum(out * seeded cotangent), through the reference's
    own recurrences.  WKV: zero initial state (the reference op has none) and
    only the outputs y carry gradient.  ROSA: the ungated read of the CUDA op is
    the reference recurrence with sigmoid(read_gate) = 1 (read_gate = 80), and
    only the reads carry gradient (the final memory is non-differentiable in
    rosa_cuda.py:117)."""
    out = {}
    wcases = [("w_n40", 2, 32, 2, 40, 31), ("w_n16", 1, 48, 3, 16, 32), ("w_n64", 1, 16, 2, 64, 33),
              ("w_n32_t20", 2, 20, 1, 32, 34)]
    for name, B, T, H, N, seed in wcases:
        ins = wkv_op_inputs(B, T, H, N, seed=seed)
        dy = np.random.default_rng(seed + 1000).standard_normal((B, T, H, N), dtype=np.float32)
        xs = [t(ins[k]).requires_grad_(True) for k in ("r", "w", "k", "v", "a", "b")]
        y, _ = RWKV7TimeMix._torch_recurrence(*xs, torch.zeros(B, H, N, N))
        gr = torch.autograd.grad((y * t(dy)).sum(), xs)
        for k, g in zip(("r", "w", "k", "v", "a", "b"), gr):
            out[f"{name}.{k}"] = ins[k]
            out[f"{name}.d{k}"] = g.numpy()
        out[f"{name}.dy"] = dy
        out[f"{name}.y"] = y.detach().numpy()
    rcases = [("r_r32", 2, 24, 32, 41, True), ("r_r128", 1, 40, 128, 42, False),
              ("r_r12", 3, 9, 12, 43, True), ("r_r256", 1, 17, 256, 44, True)]
    for name, B, T, R, seed, st in rcases:
        ins = rosa_op_inputs(B, T, R, seed=seed, with_state=st)
        dq = np.random.default_rng(seed + 1000).standard_normal((B, T, R), dtype=np.float32)
        keys = ("cand", "write", "decay", "direction", "m0")
        xs = {k: t(ins[k]).requires_grad_(True) for k in keys}
        gate = torch.full((B, T, R), 80.0)
        read, _ = ROSAMemory._reference_recurrence(xs["cand"], xs["write"], gate, xs["decay"],
                                                   xs["direction"], xs["m0"])
        gr = torch.autograd.grad((read * t(dq)).sum(), [xs[k] for k in keys])
        for k, g in zip(keys, gr):
            out[f"{name}.{k}"] = ins[k]
            out[f"{name}.d{k}"] = g.numpy()
        out[f"{name}.dq"] = dq
        out[f"{name}.read"] = read.detach().numpy()
    np.savez_compressed(HERE / "grads_cases.npz", **out)


def ref_model(cfg_kwargs, weights):
    cfg = RefConfig(**cfg_kwargs, use_cuda_kernel=False, use_rosa_scan=False)
    model = YufMusicGen(cfg).eval()
    model.load_state_dict({k: t(v) for k, v in weights.items()}, strict=True)
    return model


def greedy(model, prompt, n):
    with torch.no_grad():
        logits, st = model(t(prompt))
        last = logits[:, -1]
        toks, logs = [], []
        for _ in range(n):
            tok = torch.argmax(last, dim=-1)
            toks.append(tok)
            last, st = model.step(tok, st)
            logs.append(last)
    return torch.stack(toks, 1).numpy(), torch.stack(logs, 1).numpy()


def model_case(name, cfg_kwargs, seed, recipe, ids, n_greedy, keep_positions=None, regions_T=0):
    cfg = C.ModelConfig(**cfg_kwargs)
    weights = init_weights(cfg, seed, recipe)
    model = ref_model(cfg_kwargs, weights)
    out = {"ids": ids}
    with torch.no_grad():
        logits, _ = model(t(ids))
    logits = logits.numpy()
    if keep_positions is None:
        out["logits"] = logits
    else:
        out["positions"] = np.asarray(keep_positions, np.int64)
        out["logits"] = logits[:, keep_positions]
    if n_greedy:
        toks, logs = greedy(model, ids, n_greedy)
        out["greedy_tokens"] = toks
        out["greedy_logits"] = logs
    if regions_T:
        # Per-layer regions of a short prefill, the region names of
        # vulkan/scripts/dump_reference_step.py:186-322.
        short = ids[:, :regions_T]
        caps = {}
        hooks = []
        for li, blk in enumerate(model.blocks):
            def tm_hook(mod, inp, outp, li=li):
                caps[f"L{li}.tm_out"] = outp[0].detach().numpy()
                caps[f"L{li}.S"] = outp[1].memory.detach().numpy()
                caps[f"L{li}.prev"] = outp[1].previous.detach().numpy()
            def ro_hook(mod, inp, outp, li=li):
                caps[f"L{li}.rosa_out"] = outp[0].detach().numpy()
                caps[f"L{li}.m"] = outp[1].detach().numpy()
            def blk_hook(mod, inp, outp, li=li):
                caps[f"L{li}.h3"] = outp[0].detach().numpy()
            hooks.append(blk.time_mix.register_forward_hook(tm_hook))
            hooks.append(blk.rosa.register_forward_hook(ro_hook))
            hooks.append(blk.register_forward_hook(blk_hook))
        with torch.no_grad():
            lg, _ = model(t(short))
        for h in hooks:
            h.remove()
        caps["logits"] = lg.numpy()
        for k, v in caps.items():
            out[f"regions.{k}"] = v
        out["regions_T"] = np.int64(regions_T)
    meta = dict(seed=seed, recipe=recipe, **cfg_kwargs)
    out["meta_keys"] = np.array(list(meta.keys()))
    out["meta_vals"] = np.array([str(v) for v in meta.values()])
    np.savez_compressed(HERE / f"model_{name}.npz", **out)


def model_long_case(name, cfg_kwargs, seed, recipe, ids, positions, layers):
    """A benchmark-size prefill (the shapes that take the time-parallel WKV-7 and
    ROSA scans inside the model): the logits at a few positions and, for a few
    layers, what the reference's two recurrences returned -- the WKV-7 output y
    (at the kept positions) and final state S, the gated ROSA read (kept
    positions) and final memory m -- plus the block output h3 (kept positions).
    The recurrences are observed by wrapping the reference's own static methods
    (RWKV7TimeMix._torch_recurrence, ROSAMemory._reference_recurrence), which
    YufMusicGen.forward calls once per layer in layer order."""
    cfg = C.ModelConfig(**cfg_kwargs)
    weights = init_weights(cfg, seed, recipe)
    model = ref_model(cfg_kwargs, weights)
    pos = np.asarray(positions, np.int64)
    caps, calls = {}, {"wkv": 0, "rosa": 0}
    wkv_orig = RWKV7TimeMix._torch_recurrence
    rosa_orig = ROSAMemory._reference_recurrence

    def wkv(*a):
        y, S = wkv_orig(*a)
        li = calls["wkv"]
        calls["wkv"] += 1
        if li in layers:
            caps[f"L{li}.y"] = y[:, pos].numpy()
            caps[f"L{li}.S"] = S.numpy()
        return y, S

    def rosa(*a):
        read, m = rosa_orig(*a)
        li = calls["rosa"]
        calls["rosa"] += 1
        if li in layers:
            caps[f"L{li}.read"] = read[:, pos].numpy()
            caps[f"L{li}.m"] = m.numpy()
        return read, m

    hooks = []
    for li, blk in enumerate(model.blocks):
        if li in layers:
            def blk_hook(mod, inp, outp, li=li):
                caps[f"L{li}.h3"] = outp[0][:, pos].detach().numpy()
            hooks.append(blk.register_forward_hook(blk_hook))
    RWKV7TimeMix._torch_recurrence = staticmethod(wkv)
    ROSAMemory._reference_recurrence = staticmethod(rosa)
    try:
        with torch.no_grad():
            logits, _ = model(t(ids))
    finally:
        RWKV7TimeMix._torch_recurrence = staticmethod(wkv_orig)
        ROSAMemory._reference_recurrence = staticmethod(rosa_orig)
        for h in hooks:
            h.remove()
    assert calls["wkv"] == cfg.n_layers and calls["rosa"] == cfg.n_layers
    out = {"ids": ids, "positions": pos, "layers": np.asarray(layers, np.int64),
           "logits": logits[:, pos].numpy()}
    for k, v in caps.items():
        out[f"regions.{k}"] = v
    meta = dict(seed=seed, recipe=recipe, **cfg_kwargs)
    out["meta_keys"] = np.array(list(meta.keys()))
    out["meta_vals"] = np.array([str(v) for v in meta.values()])
    np.savez_compressed(HERE / f"model_{name}.npz", **out)


def long_cases():
    """Benchmark config 3 at its full size (0.1B model, B2 x T2048, the ids the
    benchmark prefills) and the 24-layer config-5 geometry (d1024, N = 64,
    R = 256) at B2 x T512."""
    ids3 = zipf_ids(2, 2048, seed=1, vocab=20000)
    model_long_case("c3_full", C.BASE_0P1B, seed=1, recipe="baseline", ids=ids3,
                    positions=[0, 63, 64, 255, 1024, 2047], layers=[0, 7, 13])
    ids5 = zipf_ids(2, 512, seed=5, vocab=20000)
    model_long_case("c5_geometry", C.LONG_1K, seed=2, recipe="baseline", ids=ids5,
                    positions=[0, 255, 256, 511], layers=[0, 12, 23])


def sampler_cases():
    """The reference's sampled decode rule, drawn by the reference itself:
    ``sample_token`` of yufmusicgen/cli/generate.py:45-56 (temperature, sort,
    top-p cut, ``torch.multinomial`` on the CPU MT19937 stream after
    ``torch.manual_seed``), applied to rows masked as the reference's loop masks
    them (generate.py:142-149: ids below MIDI_OFFSET = 260 excluded, EOS = 2
    selectable from step MIN_MIDI_TOKENS_BEFORE_EOS = 16 on).  The CLI module
    imports the MIDI codec packages (miditok, symusic), which are absent here
    and unused by ``sample_token``; empty stand-ins let the import succeed.
    Stored per case: the masked logits rows (in call order), the knobs, the seed
    and the tokens (logits are float16-representable and stored as float16, so
    the float32 rows are exact); plus raw Exp(1) draws of the generator (the
    multinomial's per-element keys)."""
    import types

    class _Stub(types.ModuleType):
        def __getattr__(self, name):
            if name.startswith("__"):
                raise AttributeError(name)
            return type(name, (), {})

    for name in ("miditok", "symusic", "miditok.classes", "symusic.core"):
        sys.modules.setdefault(name, _Stub(name))
    from yufmusicgen.cli.generate import MIN_MIDI_TOKENS_BEFORE_EOS, sample_token
    from yufmusicgen.tokenizer import EOS, MIDI_OFFSET

    out = {}
    cases = [  # name, vocab, rows, temperature, top_p, seed, logit scale
        ("v20000_t1_p095", 20000, 20, 1.0, 0.95, 1337, 3.0),
        ("v20000_t08_p05", 20000, 12, 0.8, 0.5, 7, 4.0),
        ("v673_t13_p1", 673, 48, 1.3, 1.0, 2024, 2.0),
        ("v673_t1_p09_peaked", 673, 40, 1.0, 0.9, 5, 8.0),
        ("v673_greedy", 673, 8, 0.0, 0.95, 11, 2.0),
    ]
    for name, V, rows, temp, top_p, seed, scale in cases:
        g = torch.Generator().manual_seed(seed + 99)
        # fp16-representable values, stored as float16 (exact as float32)
        raw = (torch.randn(rows, V, generator=g) * scale).half().float()
        masked = torch.full_like(raw, float("-inf"))
        masked[:, MIDI_OFFSET:] = raw[:, MIDI_OFFSET:]
        for i in range(rows):
            if i >= MIN_MIDI_TOKENS_BEFORE_EOS:
                masked[i, EOS] = raw[i, EOS]
        torch.manual_seed(seed)
        toks = [int(sample_token(masked[i:i + 1], temp, top_p).item()) for i in range(rows)]
        out[f"{name}.logits"] = masked.numpy().astype(np.float16)
        out[f"{name}.tokens"] = np.asarray(toks, np.int64)
        out[f"{name}.knobs"] = np.asarray([temp, top_p], np.float64)
        out[f"{name}.seed"] = np.int64(seed)
    torch.manual_seed(1337)
    out["exp_draws_seed1337"] = torch.empty(3000).exponential_().numpy()
    # the reference's whole sampled loop on the 0.1B model (config-4 prompt,
    # temperature 1.0, top-p 0.95, seed 1337), written out as run_generation
    # runs it (generate.py:130-152) around the reference's own sample_token and
    # YufMusicGen.forward / .step; per step also the margin of the draw: the
    # winning key p/q over the runner-up's, minus 1 (keys replayed from the
    # generator state before the draw)
    cfg = C.ModelConfig(**C.BASE_0P1B)
    model = ref_model(C.BASE_0P1B, init_weights(cfg, 1, "baseline"))
    prompt = zipf_ids(1, 64, seed=4, vocab=cfg.vocab_size)
    torch.manual_seed(1337)
    toks, margins = [], []
    with torch.no_grad():
        logits, st = model(t(prompt))
        logits = logits[:, -1]
        for index in range(48):
            allowed = torch.full_like(logits, float("-inf"))
            allowed[:, MIDI_OFFSET:] = logits[:, MIDI_OFFSET:]
            if index >= MIN_MIDI_TOKENS_BEFORE_EOS:
                allowed[:, EOS] = logits[:, EOS]
            state = torch.get_rng_state()
            x = allowed / 1.0
            sl, _ = torch.sort(x, descending=True, dim=-1)
            pr = torch.softmax(sl, -1)
            sl = sl.masked_fill(torch.cumsum(pr, -1) - pr > 0.95, float("-inf"))
            keys = torch.softmax(sl, -1) / torch.empty_like(sl).exponential_()
            top2 = torch.topk(keys[0], 2).values
            margins.append(float(top2[0] / top2[1] - 1))
            torch.set_rng_state(state)
            token = sample_token(allowed, 1.0, 0.95)
            if int(token.item()) == EOS:
                break
            toks.append(int(token.item()))
            logits, st = model.step(token, st)
    out["decode.prompt"] = prompt
    out["decode.tokens"] = np.asarray(toks, np.int64)
    out["decode.margins"] = np.asarray(margins, np.float64)
    out["cases"] = np.array([c[0] for c in cases])
    np.savez_compressed(HERE / "sampler_torch_cpu.npz", **out)


def state_test_case():
    """The reference's own sequence-vs-step test (tests/test_model_state.py:9-28),
    with the reference recurrence selected (use_rosa_scan=False)."""
    torch.manual_seed(7)
    cfg = RefConfig(**C.STATE_TEST, use_cuda_kernel=False, use_rosa_scan=False)
    model = YufMusicGen(cfg).eval()
    tokens = torch.randint(0, cfg.vocab_size, (1, 6))
    with torch.no_grad():
        full, _ = model(tokens)
        st = None
        steps = []
        for i in range(tokens.shape[1]):
            lg, st = model.step(tokens[:, i], st)
            steps.append(lg)
    sd = {k: v.numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(
        HERE / "model_state_test.npz",
        ids=tokens.numpy(), logits=full.numpy(), stepped=torch.stack(steps, 1).numpy(),
        **{f"w.{k}": v for k, v in sd.items()},
    )


def greedy256_case():
    """The north star's greedy bar on the 0.1B model (benchmark configs 3/4):
    two 64-token config-4 prompts, 256 greedy decode steps through
    ``YufMusicGen.forward`` + ``.step`` (yufmusicgen/model.py:406-431).  Stored:
    the tokens, each step's top-1 minus top-2 logit margin (how far a step is
    from a tie) and the full logits of the first and last step."""
    cfg = C.ModelConfig(**C.BASE_0P1B)
    weights = init_weights(cfg, 1, "baseline")
    model = ref_model(C.BASE_0P1B, weights)
    ids = zipf_ids(2, 64, seed=4, vocab=cfg.vocab_size)
    n = 256
    with torch.no_grad():
        logits, st = model(t(ids))
        last = logits[:, -1]
        toks, gaps, keep = [], [], {}
        for i in range(n):
            top2 = torch.topk(last, 2, dim=-1).values
            gaps.append(top2[:, 0] - top2[:, 1])
            tok = torch.argmax(last, dim=-1)
            toks.append(tok)
            last, st = model.step(tok, st)
            if i in (0, n - 1):
                keep[i] = last.numpy().copy()
    np.savez_compressed(
        HERE / "greedy256_base0p1b.npz", ids=ids, tokens=torch.stack(toks, 1).numpy(),
        margins=torch.stack(gaps, 1).numpy(), logits_step0=keep[0], logits_last=keep[n - 1],
        meta_keys=np.array(["seed", "recipe", "steps"]), meta_vals=np.array(["1", "baseline", str(n)]))


def dropin_case():
    """What the reference op wrapper hands its CUDA op: ``_pad_inputs`` of
    yufmusicgen/cuda_ops.py:160-186 on T not a multiple of 16, and the CPU
    recurrence's y and final state for the unpadded inputs (zero state)."""
    from yufmusicgen import cuda_ops as ref_ops

    out = {}
    for name, B, T, H, N, seed in (("n40_t21", 2, 21, 3, 40, 31), ("n64_t5", 1, 5, 2, 64, 32),
                                   ("n16_t37", 2, 37, 2, 16, 33)):
        ins = wkv_op_inputs(B, T, H, N, seed=seed)
        args = [t(ins[k]) for k in ("r", "w", "k", "v", "a", "b")]
        padded, length = ref_ops._pad_inputs(*args)
        assert length == T
        y, sT = RWKV7TimeMix._torch_recurrence(*args, torch.zeros(B, H, N, N))
        for k, x in zip(("r", "w", "k", "v", "a", "b"), padded):
            out[f"{name}.{k}_padded"] = x.numpy()
            out[f"{name}.{k}"] = ins[k]
        out[f"{name}.length"] = np.array(length)
        out[f"{name}.y"] = y.numpy()
        out[f"{name}.sT"] = sT.numpy()
    np.savez_compressed(HERE / "dropin_pad_cases.npz", **out)


def main():
    wkv_cases()
    rosa_cases()
    state_test_case()
    model_case("tiny", C.TINY, seed=0, recipe="perturbed", ids=tiny_ids(2, 256, seed=0),
               n_greedy=64, regions_T=16)
    model_case("tiny_baseline", C.TINY, seed=0, recipe="baseline", ids=tiny_ids(2, 64, seed=3),
               n_greedy=16)
    ids3 = zipf_ids(1, 24, seed=1, vocab=20000, byte_prefix=8)
    model_case("base0p1b", C.BASE_0P1B, seed=1, recipe="baseline", ids=ids3, n_greedy=8,
               keep_positions=[0, 7, 8, 23])
    c5 = dict(C.LONG_1K, n_layers=2)
    ids5 = zipf_ids(1, 12, seed=2, vocab=20000, byte_prefix=0)
    model_case("long1k_2l", c5, seed=2, recipe="perturbed", ids=ids5, n_greedy=4,
               keep_positions=[0, 11])
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    if sys.argv[1:] == ["grads"]:
        grad_cases()
    elif sys.argv[1:] == ["long"]:
        long_cases()
    elif sys.argv[1:] == ["sampler"]:
        sampler_cases()
    elif sys.argv[1:] == ["greedy256"]:
        greedy256_case()
    elif sys.argv[1:] == ["dropin"]:
        dropin_case()
    else:
        main()
        grad_cases()
        greedy256_case()
        long_cases()
        dropin_case()
        sampler_cases()
