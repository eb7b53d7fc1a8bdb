"""Oracle restatement of the packed RWKV-7 decode forward (NumPy fp32, CPU).

Test infrastructure: see ``oracle/__init__.py``.

Restates, step for step and in fp32 activations:

* ``tmix_one_fused``        — ``rwkv_ssd/runtime/rwkv7_linear.py:125-356``
* ``cmix_one_fused``        — ``rwkv_ssd/runtime/rwkv7_linear.py:359-435``
* ``forward_block_packed``  — ``rwkv_ssd/runtime/packed_block_forward.py:76-166``
* embedding + ``ln0``       — ``rwkv_ssd/runtime/rwkv7_skeleton.py:74-81``
* ``ln_out`` + packed head  — ``rwkv_ssd/backends/rwkv7_forward.py:791-809``
* greedy argmax (first max) — ``rwkv_ssd/runtime/sampling.py:161-163``
* zero state layout         — ``rwkv_ssd/runtime/rwkv7_skeleton.py:121-131``

Packed GEMVs run through ``oracle.kernels`` (the restated C kernels, or the
reference's own C kernels with ``impl="reference"``).

The same class runs one rank's shard of a tensor-parallel split (heads, FFN
rows and vocabulary rows, as ``rwkv_b200.tp.shard_pack`` makes it): widths are
read from the pack, ``reduce`` sums the output and FFN value projections over
the ranks and ``argmax`` picks the global first maximum.  With the defaults
(identity, ``np.argmax``) and a full pack it is the single-device restatement.

A *pack* is a mapping ``name -> entry`` where ``entry`` has ``codec``
(``"sg8"``, ``"lut2"`` or ``"none"``), ``payload`` (wire bytes, or an fp32
array for ``"none"``) and ``shape`` (checkpoint shape).
"""

from __future__ import annotations

import numpy as np

from oracle import codec as oc
from oracle import kernels as ok

LN_EPS = 1e-5          # F.layer_norm default (packed_block_forward.py:94-98)
GN_EPS = 64e-5         # rwkv7_linear.py:344
DECAY_SCALE = np.float32(0.606531)  # rwkv7_linear.py:314


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = LN_EPS) -> np.ndarray:
    x = x.astype(np.float32)
    mu = x.mean(dtype=np.float32)
    var = ((x - mu) ** 2).mean(dtype=np.float32)
    return ((x - mu) / np.sqrt(var + np.float32(eps)) * w + b).astype(np.float32)


class OracleRWKV7:
    """Token-by-token RWKV-7 decode over a packed model, on the CPU."""

    def __init__(self, pack, *, n_layer: int, n_embd: int, head_size: int,
                 impl: str = "oracle", reduce=None, argmax=None):
        self.pack = pack
        self.L = int(n_layer)
        self.C = int(n_embd)
        self.N = int(head_size)
        # attention heads held (all of them, or a tensor-parallel shard)
        rk = pack.get("blocks.0.att.r_k")
        self.H = int(rk.shape[0]) if rk is not None else self.C // self.N
        self.Ca = self.H * self.N
        self.impl = impl
        self.reduce = reduce if reduce is not None else (lambda v: v)
        self.argmax = argmax if argmax is not None else (lambda logits: int(np.argmax(logits)))
        self._dense: dict[str, np.ndarray] = {}
        self.vocab = int(pack["head.weight"].shape[0])

    # ---------------------------------------------------------------- params
    def vec(self, name: str) -> np.ndarray:
        """A skeleton tensor as a flat fp32 vector (decoded when packed)."""
        if name not in self._dense:
            e = self.pack[name]
            if e.codec == "none":
                v = np.asarray(e.payload, dtype=np.float32).reshape(-1)
            elif e.codec == "sg8":
                v = oc.decode_sg8(e.payload, int(np.prod(e.shape)))
            else:
                v = oc.decode_lut2_grouped(e.payload, tuple(e.shape)).reshape(-1)
            self._dense[name] = v
        return self._dense[name]

    def gemv(self, name: str, x: np.ndarray) -> np.ndarray:
        e = self.pack[name]
        out_f, in_f = int(e.shape[0]), int(e.shape[1])
        return ok.packed_gemv(e.payload, x, out_f, in_f, self.impl)

    def zero_state(self) -> list[np.ndarray]:
        st: list[np.ndarray] = []
        for _ in range(self.L):
            st.append(np.zeros(self.C, np.float32))
            st.append(np.zeros((self.H, self.N, self.N), np.float32))
            st.append(np.zeros(self.C, np.float32))
        return st

    # ------------------------------------------------------------------ ops
    def embed(self, token: int) -> np.ndarray:
        e = self.pack["emb.weight"]
        V, C = int(e.shape[0]), int(e.shape[1])
        if not 0 <= token < V:
            raise ValueError(f"token id {token} is outside the vocabulary")
        if e.codec == "sg8":
            g, _, _ = oc.sg8_parse(e.payload, V * C)
            row = self._sg8_rows(e.payload, V * C, token * C, C)
        elif e.codec == "none":
            row = np.asarray(e.payload, np.float32).reshape(V, C)[token]
        else:
            row = oc.decode_lut2_grouped(e.payload, (V, C))[token]
        return layer_norm(row, self.vec("blocks.0.ln0.weight"), self.vec("blocks.0.ln0.bias"))

    @staticmethod
    def _sg8_rows(blob, numel: int, start: int, count: int) -> np.ndarray:
        """Decode elements ``[start, start+count)`` of an SG8 tensor with the
        exact ``pack_codec.py:174-182`` arithmetic."""
        g, scales, quant = oc.sg8_parse(blob, numel)
        idx = np.arange(start, start + count)
        grp = idx // g
        mn = scales[grp, 0]
        delta = (scales[grp, 1] - mn) * np.float32(1.0 / 255.0)
        return (quant[idx].astype(np.float32) * delta + mn).astype(np.float32)

    def tmix(self, layer: int, x: np.ndarray, x_prev: np.ndarray, v_first,
             S: np.ndarray):
        """``tmix_one_fused`` (rwkv7_linear.py:125-356). Returns
        ``(out, new_x_prev, new_S, v_first)``."""
        H, N, C = self.H, self.N, self.Ca
        p = f"blocks.{layer}.att."
        xx = x_prev - x
        xr = x + xx * self.vec(p + "x_r")
        xw = x + xx * self.vec(p + "x_w")
        xk = x + xx * self.vec(p + "x_k")
        xv = x + xx * self.vec(p + "x_v")
        xa = x + xx * self.vec(p + "x_a")
        xg = x + xx * self.vec(p + "x_g")
        r = self.gemv(p + "receptance.weight", xr)
        k = self.gemv(p + "key.weight", xk)
        v = self.gemv(p + "value.weight", xv)

        names = ["w1", "w2", "a1", "a2", "g1", "g2"] + (["v1", "v2"] if layer != 0 else [])
        ents = [self.pack[p + n] for n in names]
        if all(e.codec == "sg8" for e in ents) and self.Ca == self.C:
            ranks = [ents[0].shape[1], ents[2].shape[1], ents[4].shape[1],
                     ents[6].shape[1] if layer != 0 else 0]
            xs = [xw, xa, xg] + ([xv] if layer != 0 else [])
            w, a, g, v_gate = ok.sg8_tmix_adapters([e.payload for e in ents], xs,
                                                   self.vec(p + "a0"), C, ranks, self.impl)
        else:
            def xw_(n, vec):
                W = self.vec(p + n).reshape(self.pack[p + n].shape)
                return (vec @ W).astype(np.float32)
            w = xw_("w2", np.tanh(xw_("w1", xw)).astype(np.float32))
            a = _sigmoid(self.vec(p + "a0") + xw_("a2", xw_("a1", xa)))
            g = xw_("g2", _sigmoid(xw_("g1", xg)))
            v_gate = xw_("v2", xw_("v1", xv)) if layer != 0 else None

        kk = (k * self.vec(p + "k_k")).reshape(H, N)
        nrm = np.sqrt((kk * kk).sum(axis=1, dtype=np.float32))
        kk = (kk / np.maximum(nrm, np.float32(1e-12))[:, None]).reshape(C).astype(np.float32)
        k = k * (np.float32(1.0) + (a - np.float32(1.0)) * self.vec(p + "k_a"))
        if layer == 0:
            v_first = v
        else:
            v = v + (v_first - v) * _sigmoid(self.vec(p + "v0") + v_gate)
        w = np.exp(-DECAY_SCALE * _sigmoid(self.vec(p + "w0") + w)).astype(np.float32)

        kkh = kk.reshape(H, N)
        kah = (kk * a).reshape(H, N)
        sa = np.einsum("hij,hj->hi", S, -kkh).astype(np.float32)
        S = (S * w.reshape(H, 1, N) + sa[:, :, None] * kah[:, None, :]
             + v.reshape(H, N, 1) * k.reshape(H, 1, N)).astype(np.float32)
        y = np.einsum("hij,hj->hi", S, r.reshape(H, N)).astype(np.float32)

        mu = y.mean(axis=1, keepdims=True, dtype=np.float32)
        var = ((y - mu) ** 2).mean(axis=1, keepdims=True, dtype=np.float32)
        y = ((y - mu) / np.sqrt(var + np.float32(GN_EPS))).reshape(C)
        y = y * self.vec(p + "ln_x.weight") + self.vec(p + "ln_x.bias")
        bonus = (r * k * self.vec(p + "r_k")).reshape(H, N).sum(axis=1, keepdims=True, dtype=np.float32)
        y = (y + (bonus * v.reshape(H, N)).reshape(C)).astype(np.float32)
        out = self.reduce(self.gemv(p + "output.weight", (y * g).astype(np.float32)))
        return out, x, S, v_first

    def cmix(self, layer: int, x: np.ndarray, x_prev: np.ndarray):
        """``cmix_one_fused`` (rwkv7_linear.py:359-435)."""
        p = f"blocks.{layer}.ffn."
        k = x + (x_prev - x) * self.vec(p + "x_k")
        ke, ve = self.pack[p + "key.weight"], self.pack[p + "value.weight"]
        if ke.codec == "sg8" and ve.codec == "sg8":
            out = ok.sg8_cmix(ke.payload, ve.payload, k, ke.shape[0], ke.shape[1],
                              ve.shape[0], ve.shape[1], self.impl)
        else:
            h = self.gemv(p + "key.weight", k)
            h = np.maximum(h, np.float32(0.0)) ** 2
            out = self.gemv(p + "value.weight", h.astype(np.float32))
        return self.reduce(out), x

    def block(self, layer: int, x: np.ndarray, state: list, v_first):
        """``forward_block_packed`` (packed_block_forward.py:76-166)."""
        b = f"blocks.{layer}."
        xx = layer_norm(x, self.vec(b + "ln1.weight"), self.vec(b + "ln1.bias"))
        out, state[3 * layer], state[3 * layer + 1], v_first = self.tmix(
            layer, xx, state[3 * layer], v_first, state[3 * layer + 1])
        x = (x + out).astype(np.float32)
        xx = layer_norm(x, self.vec(b + "ln2.weight"), self.vec(b + "ln2.bias"))
        out, state[3 * layer + 2] = self.cmix(layer, xx, state[3 * layer + 2])
        return (x + out).astype(np.float32), v_first

    def head(self, x: np.ndarray) -> np.ndarray:
        x = layer_norm(x, self.vec("ln_out.weight"), self.vec("ln_out.bias"))
        return self.gemv("head.weight", x)

    def forward_token(self, token: int, state: list) -> np.ndarray:
        x = self.embed(int(token))
        v_first = None
        for layer in range(self.L):
            x, v_first = self.block(layer, x, state, v_first)
        return self.head(x)

    def greedy(self, prompt: list[int], n_new: int, state=None):
        """Prompt token by token, then ``n_new`` greedy tokens.

        Returns ``(generated_ids, logits[len(prompt)+n_new-1, V], state)``:
        one logits row per forward pass (the last prompt token's row picks
        the first generated id).
        """
        st = self.zero_state() if state is None else state
        rows = []
        logits = None
        for t in prompt:
            logits = self.forward_token(t, st)
            rows.append(logits)
        ids = []
        for i in range(n_new):
            nxt = self.argmax(logits)
            ids.append(nxt)
            if i + 1 < n_new:
                logits = self.forward_token(nxt, st)
                rows.append(logits)
        return ids, np.stack(rows), st
