"""Ternary K/V oracle (numpy / torch on CPU; TEST INFRASTRUCTURE ONLY).

Restates sparse-ai's ternary path:
* ``quantize``  -- TernaryQuantize.forward (src/llama_surgery/surgery.py:15-28): per row,
  scale = mean |x| (fp32), value +1 where x > scale / 2, -1 where x < -scale / 2, else 0;
* ``pack`` / ``unpack`` -- pack_ternary / unpack_ternary (:35-75): codes 1 (+1), 2 (-1), 0,
  16 per int32, value i in bits [2i, 2i + 2);
* ``ternary_attention`` -- the math of ternary_ultrametric_attention_triton (kernel.py:147-249,
  348-418) with shift_size 0: K/V = code x scale rounded to fp16; query block m (of
  min(128, N) tokens) attends key block n <= m when the routes agree on the first req_depth
  levels, n == 0, or m - n <= ceil(local_window / block); token-level causal mask; softmax
  at scale 1/sqrt(D), computed here in fp64.
"""

from __future__ import annotations

import math

import numpy as np
import torch


def quantize(x: np.ndarray):
    """(..., D) -> (codes in {-1, 0, 1} as float32, scale (...) float32)."""
    xf = np.asarray(x, dtype=np.float32)
    scale = np.abs(xf).mean(-1, dtype=np.float32)
    thr = np.float32(0.5) * scale[..., None]
    codes = np.where(xf > thr, 1.0, np.where(xf < -thr, -1.0, 0.0)).astype(np.float32)
    return codes, scale


def pack(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes)
    m = np.where(c == 1.0, 1, np.where(c == -1.0, 2, 0)).astype(np.int64)
    m = m.reshape(*c.shape[:-1], c.shape[-1] // 16, 16)
    words = np.zeros(m.shape[:-1], dtype=np.int64)
    for i in range(16):
        words |= m[..., i] << (2 * i)
    return words.astype(np.uint32).view(np.int32)


def unpack(packed: np.ndarray) -> np.ndarray:
    w = np.asarray(packed).view(np.uint32).astype(np.int64)
    vals = np.stack([(w >> (2 * i)) & 3 for i in range(16)], axis=-1)
    out = np.where(vals == 1, 1.0, np.where(vals == 2, -1.0, 0.0)).astype(np.float32)
    return out.reshape(*w.shape[:-1], w.shape[-1] * 16)


def ternary_attention(q, k_packed, v_packed, k_scale, v_scale, router, local_window=128, req_depth=2):
    Z, H, N, D = q.shape
    block = min(128, N)
    nb = -(-N // block)
    k = torch.from_numpy(unpack(k_packed) * np.asarray(k_scale)[..., None]).half().double()
    v = torch.from_numpy(unpack(v_packed) * np.asarray(v_scale)[..., None]).half().double()
    r = np.zeros((Z, H, nb, router.shape[-1]), dtype=np.int64)
    r[:, :, :min(nb, router.shape[2])] = np.asarray(router)[:, :, :nb]
    lwb = math.ceil(local_window / block)
    out = torch.zeros(Z, H, N, D, dtype=torch.float64)
    scale = 1.0 / math.sqrt(D)
    qd = torch.as_tensor(q).double()
    for z in range(Z):
        for h in range(H):
            bm = np.zeros((nb, nb), dtype=bool)
            for m in range(nb):
                for n in range(m + 1):
                    match = (r[z, h, m, :req_depth] == r[z, h, n, :req_depth]).all()
                    bm[m, n] = bool(match) or n == 0 or (m - n) <= lwb
            tm = torch.from_numpy(np.repeat(np.repeat(bm, block, 0), block, 1)[:N, :N])
            tm &= torch.tril(torch.ones(N, N, dtype=torch.bool))
            s = (qd[z, h] @ k[z, h].T) * scale
            s = s.masked_fill(~tm, float("-inf"))
            out[z, h] = torch.softmax(s, -1) @ v[z, h]
    return out
