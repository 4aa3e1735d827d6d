"""numpy restatement of ``YufMusicGen`` (test oracle).

Follows the reference's fp32 CPU path with ``use_cuda_kernel=False,
use_rosa_scan=False`` -- the recipe of ``vulkan/scripts/dump_reference_step.py
:190-196``, and the only path whose sequence and step forms agree (the
``torch.scan`` ROSA path drops the read-gate sigmoid, yufmusicgen/model.py:234,
258, 327).

State layout per layer, as the reference carries it (model.py:29-37):
``prev [B, d]`` (the LayerNorm'd block input of the last token),
``S [B, H, N, N]`` (row i = value, column j = key), ``m [B, R]``.
"""

from __future__ import annotations

import numpy as np

from .scans import rosa_scan, wkv7_scan

F32 = np.float32


def _ln(x, w, b, eps=1e-5):
    # nn.LayerNorm default eps (yufmusicgen/model.py:78, 348-352, 388)
    mean = x.mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    xc = x - mean
    var = (xc.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(F32)
    return (xc / np.sqrt(var + F32(eps)) * w + b).astype(F32)


def _linear(x, w, b=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    return y.astype(F32)


def _sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(F32)


def _normalize(x, eps=1e-12):
    n = np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True)).astype(F32)
    return (x / np.maximum(n, F32(eps))).astype(F32)


class OracleModel:
    """Reference-semantics forward/step over a weight dict (reference names)."""

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self.w = {k: np.asarray(v, F32) for k, v in weights.items()}

    def initial_state(self, B):
        c = self.cfg
        return [
            dict(
                prev=np.zeros((B, c.d_model), F32),
                S=np.zeros((B, c.n_heads, c.head_size, c.head_size), F32),
                m=np.zeros((B, c.rosa_size), F32),
            )
            for _ in range(c.n_layers)
        ]

    # RWKV7TimeMix._inputs_impl, yufmusicgen/model.py:97-131
    def timemix_inputs(self, i, x, prev):
        W = self.w
        p = f"blocks.{i}.time_mix."
        c = self.cfg
        Bn, T, d = x.shape
        shifted = np.concatenate([prev[:, None], x[:, :-1]], axis=1)
        delta = x - shifted
        xr = x + delta * W[p + "mix_r"]
        xw = x + delta * W[p + "mix_w"]
        xk = x + delta * W[p + "mix_k"]
        xv = x + delta * W[p + "mix_v"]
        xa = x + delta * W[p + "mix_a"]
        xg = x + delta * W[p + "mix_g"]
        r = _linear(xr, W[p + "receptance.weight"])
        w = (W[p + "w0"] + np.tanh(xw @ W[p + "w1"]) @ W[p + "w2"]).astype(F32)
        k = _linear(xk, W[p + "key.weight"])
        v = _linear(xv, W[p + "value.weight"])
        a = _sigmoid(W[p + "a0"] + (xa @ W[p + "a1"]) @ W[p + "a2"])
        g = _sigmoid((xg @ W[p + "g1"]) @ W[p + "g2"])
        H, N = c.n_heads, c.head_size
        kk = _normalize((k * W[p + "k_k"]).reshape(Bn, T, H, N))
        k_adj = (k * (1.0 + (a - 1.0) * W[p + "k_a"])).reshape(Bn, T, H, N).astype(F32)
        a_h = a.reshape(Bn, T, H, N)
        return dict(
            r=r.reshape(Bn, T, H, N), w=w.reshape(Bn, T, H, N), k=k_adj,
            v=v.reshape(Bn, T, H, N), a=-kk, b=(kk * a_h).astype(F32), g=g,
        )

    def block(self, i, x, st, regions=None):
        W = self.w
        p = f"blocks.{i}."
        c = self.cfg
        Bn, T, d = x.shape
        # YufBlock.forward, yufmusicgen/model.py:365-378
        xt = _ln(x, W[p + "norm_time.weight"], W[p + "norm_time.bias"])
        ins = self.timemix_inputs(i, xt, st["prev"])
        y, S = wkv7_scan(ins["r"], ins["w"], ins["k"], ins["v"], ins["a"], ins["b"], st["S"])
        tm = p + "time_mix."
        mixed = y.reshape(Bn, T, d)
        o = _linear(_ln(mixed, W[tm + "out_norm.weight"], W[tm + "out_norm.bias"]) * ins["g"], W[tm + "output.weight"])
        x1 = (x + o).astype(F32)
        # ROSAMemory.forward with the reference recurrence, model.py:290-342
        xr = _ln(x1, W[p + "norm_rosa.weight"], W[p + "norm_rosa.bias"])
        ro = p + "rosa."
        cand = _linear(xr, W[ro + "input.weight"], W[ro + "input.bias"])
        write = _linear(xr, W[ro + "write_gate.weight"], W[ro + "write_gate.bias"])
        rgate = _linear(xr, W[ro + "read_gate.weight"], W[ro + "read_gate.bias"])
        decay = _sigmoid(W[ro + "decay"])
        direction = _normalize(W[ro + "householder"])
        read, m = rosa_scan(cand, write, rgate, decay, direction, st["m"])
        x2 = (x1 + _linear(read, W[ro + "output.weight"])).astype(F32)
        xf = _ln(x2, W[p + "norm_ffn.weight"], W[p + "norm_ffn.bias"])
        hid = _linear(xf, W[p + "ffn_in.weight"])
        silu = (hid * _sigmoid(hid)).astype(F32)
        ffn = _linear(silu * _linear(xf, W[p + "ffn_gate.weight"]), W[p + "ffn_out.weight"])
        x3 = (x2 + ffn).astype(F32)
        if regions is not None:
            regions[i] = dict(
                ln0=xt, r=ins["r"], w=ins["w"], k=ins["k"], v=ins["v"], a=ins["a"], b=ins["b"],
                g=ins["g"], y=y, S=S, o=o, h1=x1, cand=cand, write=write, read_gate=rgate,
                read=read, m=m, h2=x2, h3=x3,
            )
        return x3, dict(prev=xt[:, -1].copy(), S=S, m=m)

    def forward(self, ids, state=None, regions=None):
        """YufMusicGen.forward (model.py:406-422): logits [B, T, V] and next state."""
        ids = np.asarray(ids)
        Bn, T = ids.shape
        x = self.w["token_embedding.weight"][ids].astype(F32)
        st = state if state is not None else self.initial_state(Bn)
        nxt = []
        for i in range(self.cfg.n_layers):
            x, s = self.block(i, x, st[i], regions)
            nxt.append(s)
        h = _ln(x, self.w["final_norm.weight"], self.w["final_norm.bias"])
        logits = _linear(h, self.w["lm_head.weight"])
        return logits, nxt

    def step(self, ids, state):
        """YufMusicGen.step (model.py:424-431): logits of the single new token."""
        ids = np.asarray(ids).reshape(-1, 1)
        logits, state = self.forward(ids, state)
        return logits[:, -1], state

    def greedy(self, prompt, n_steps):
        """Prefill ``prompt`` then take ``n_steps`` argmax tokens through ``step``.

        Returns (tokens [B, n_steps], step logits [B, n_steps, V]).  The first
        token is the argmax of the prefill's last logits.
        """
        logits, st = self.forward(prompt)
        last = logits[:, -1]
        toks, logs = [], []
        for _ in range(n_steps):
            tok = np.argmax(last, axis=-1)
            toks.append(tok)
            last, st = self.step(tok, st)
            logs.append(last)
        return np.stack(toks, 1), np.stack(logs, 1)
