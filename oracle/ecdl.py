"""CPU restatement of cdl's ECDL quantizer -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` use this module, as the checker of ``csrc/ecdl.cu``; the
product never imports it.  It restates, in numpy float32, the algorithm of

* ``cdl/core/kernel/ecdl/kernel.py:34-117`` (``_ecdl_fwd``: block scale per
  scale mode, ``v = x / s``, one sampled level index per element, packing),
  ``:120-185`` (``_ecdl_bwd``: proxy-gradient coefficients, the d(kappa)
  and d(alpha) partial sums),
* ``cdl/core/kernel/ecdl/launch.py:20-95`` (block absmax, global absmax,
  ``alpha_eff``),
* ``cdl/core/kernel/primitives.py:23-70`` (``cdl_window``, ``cdl_weight``,
  ``cdl_sample``) and ``:137-187`` (``cdl_proxy_coeffs``),
* ``cdl/core/kernel/formats/spec.py`` / ``cdl/core/tables.py`` /
  ``cdl/api/format.py:7-10`` (level and gap tables) and
  ``cdl/core/kernel/formats/ordinals.py`` (nearest-level ordinals),

with the uniform numbers of Triton's ``tl.rand(seed, offset)``: Philox4x32-10
(the Random123 generator, constants below) on counter ``(offset, 0, 0, 0)``
and key ``(seed_lo, seed_hi)``, first output word, mapped to [0, 1) as
``(x < 0 ? -x - 1 : x) * 4.6566127342e-10`` on its int32 view (Triton
``python/triton/language/random.py``, 3.x).  Checked against the Random123
known-answer vectors in ``tests/test_ecdl_cpu.py``; the window, the sampling
probabilities, the expected level and its derivatives against the
reference's torch formulae (``cdl/core/formulae.py`` topk_cpmf_companded /
topk_q_d and their autograd gradients; ``tests/golden/cdl_window.npz``, made
by ``tests/golden/make_cdl_golden.py``); the CCDL eval round against the
reference's ``cascaded_nearest_round`` (``tests/golden/ccdl_round.npz``).

Parity of the sampled codes is statistical at the edges: an element whose
``u * z`` falls within float rounding of a cumulative boundary may pick the
neighbouring level when the weights differ in the last bit.
"""

from __future__ import annotations

import numpy as np

NVFP4, MXFP4, MXFP8 = 0, 1, 2
MODE_NVIDIA, MODE_OCP = 0, 1
TINY = np.float32(1.1754943508222875e-38)
LOG2E = np.float32(1.4426950408889634)

# ---------------------------------------------------------------------------
# Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3",
# SC 2011), as Triton's tl.rand uses it
# ---------------------------------------------------------------------------
_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32(c0, c1, c2, c3, k0, k1, rounds: int = 10):
    c = [np.asarray(x, dtype=np.uint64) & _MASK for x in (c0, c1, c2, c3)]
    k0, k1 = np.uint64(k0) & _MASK, np.uint64(k1) & _MASK
    for _ in range(rounds):
        p0 = _M0 * c[0]
        p1 = _M1 * c[2]
        c = [((p1 >> np.uint64(32)) ^ c[1] ^ k0) & _MASK, p1 & _MASK,
             ((p0 >> np.uint64(32)) ^ c[3] ^ k1) & _MASK, p0 & _MASK]
        k0 = (k0 + _W0) & _MASK
        k1 = (k1 + _W1) & _MASK
    return [x.astype(np.uint32) for x in c]


def uniform(seed: int, offsets: np.ndarray) -> np.ndarray:
    """tl.rand(seed, offsets) with the seed loaded as int32 (kernel.py:101)."""
    s32 = ((int(seed) + 2 ** 31) % 2 ** 32) - 2 ** 31  # the low 32 bits as a signed int32
    lo = s32 & 0xFFFFFFFF
    hi = 0xFFFFFFFF if s32 < 0 else 0
    zeros = np.zeros_like(offsets, dtype=np.uint64)
    x = philox4x32(offsets.astype(np.uint64), zeros, zeros, zeros, lo, hi)[0]
    xi = x.view(np.int32).astype(np.int64)
    xi = np.where(xi < 0, -xi - 1, xi)
    return xi.astype(np.float32) * np.float32(4.6566127342e-10)


# ---------------------------------------------------------------------------
# formats
# ---------------------------------------------------------------------------
def e4m3_value(byte: np.ndarray) -> np.ndarray:
    b = np.asarray(byte, dtype=np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e, m = (b >> 3) & 0xF, b & 7
    mag = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8.0) * 2.0 ** (e - 7.0))
    mag = np.where((b & 0x7F) == 0x7F, np.nan, mag)
    return (sign * mag).astype(np.float32)


def e4m3_rne(v: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3 byte, round to nearest even (inputs already within +-448)."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v).astype(np.float32)
    sign = np.where(np.signbit(v), 0x80, 0).astype(np.int64)
    bits = a.view(np.uint32).astype(np.int64)
    e32 = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    e = e32 - 127 + 7
    m3 = mant >> 20
    rem = mant & 0xFFFFF
    up = (rem > 0x80000) | ((rem == 0x80000) & (m3 & 1 == 1))
    m3 = m3 + up
    e = e + (m3 >> 3)
    m3 = m3 & 7
    normal = (e << 3) | m3
    sub = np.rint(a.astype(np.float64) * 2.0 ** 9).astype(np.int64)  # |v| < 2^-6: m * 2^-9, RNE
    byte = np.where(a >= np.float32(2.0 ** -6), normal, sub)
    return (byte | sign).astype(np.int64)


def gaps(level: np.ndarray) -> np.ndarray:
    gap = np.diff(level).astype(np.float32)
    gap = np.concatenate([gap, gap[-1:]])
    return np.where(gap == 0, np.roll(gap, 1), gap).astype(np.float32)


def e2m1_levels() -> np.ndarray:
    mag = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
    key = np.arange(16)
    return np.where(key >= 8, mag[np.clip(key - 8, 0, 7)], -mag[np.clip(7 - key, 0, 7)]).astype(np.float32)


def e4m3_levels() -> np.ndarray:
    key = np.arange(254)
    return e4m3_value(np.where(key >= 127, key - 127, 254 - key))


def q_levels(fmt: int) -> np.ndarray:
    if fmt == NVFP4:  # UE4M3 without zero: bytes 1..126
        return e4m3_value(np.arange(1, 127))
    b = np.arange(255)  # E8M0: byte 0 is the subnormal 2^-127
    return np.where(b == 0, np.float32(2.0 ** -127), np.ldexp(np.float32(1.0), b - 127)).astype(np.float32)


class Format:
    def __init__(self, fmt: int):
        self.fmt = fmt
        self.level = e4m3_levels() if fmt == MXFP8 else e2m1_levels()
        self.gap = gaps(self.level)
        self.tn = self.level.size
        self.q = q_levels(fmt)
        self.qn = self.q.size
        self.q_max = np.float32(self.q[-1])
        # a Python float in the reference (spec.py); only the nvidia mode (NVFP4, 2688) uses it
        self.f_max = float(np.abs(self.level).max()) * float(self.q.max())
        self.emax = int(np.floor(np.log2(float(np.abs(self.level).max()))))
        self.bias = 1 if fmt == NVFP4 else 0
        self.tpb = 16 if fmt == NVFP4 else 32

    def ordinal(self, v: np.ndarray) -> np.ndarray:
        if self.fmt == MXFP8:
            b = e4m3_rne(np.clip(v, -448.0, 448.0))
            return np.clip(np.where(b < 128, b + 127, 254 - b), 0, self.tn - 1)
        sgn = np.signbit(v)
        av = np.minimum(np.abs(v), np.float32(6.0))
        mag = sum((av > t).astype(np.int64) for t in (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0))
        return np.where(sgn, 7 - mag, 8 + mag)

    def q_ordinal(self, v: np.ndarray) -> np.ndarray:  # UE4M3 (nvidia mode)
        b = e4m3_rne(np.clip(v, np.float32(2.0 ** -9), np.float32(448.0)))
        return np.clip(b - 1, 0, self.qn - 1)


# ---------------------------------------------------------------------------
# the CDL window / sampler / proxy coefficients (float32 throughout)
# ---------------------------------------------------------------------------
def _window(f: Format, v, topk):
    key = f.ordinal(v)
    klev = f.level[key]
    left = np.maximum(key - 1, 0)
    kgap = np.where(v >= klev, f.gap[key], f.gap[left]).astype(np.float32)
    c = (key.astype(np.float32) + (v - klev).astype(np.float32) / kgap).astype(np.float32)
    start = np.clip(key - topk // 2, 0, f.tn - topk)
    return c, start, kgap


def _near(c, start, topk, kappa):
    t_near = np.clip(np.floor(c + np.float32(0.5)), start.astype(np.float32),
                     (start + topk - 1).astype(np.float32)).astype(np.int64)
    dn = (t_near.astype(np.float32) - c).astype(np.float32)
    m = (-kappa * dn * dn).astype(np.float32)
    return t_near, m


def _weight(c, t, t_near, m, kappa):
    d = (c - t).astype(np.float32)
    x = np.minimum((-kappa * d * d - m).astype(np.float32), np.float32(0.0))
    w = np.exp2((x * LOG2E).astype(np.float32)).astype(np.float32)
    return np.where(t == t_near, np.float32(1.0), w).astype(np.float32), d


def sample(f: Format, v, kappa, u, topk):
    kappa = np.float32(kappa)
    c, start, _ = _window(f, v, topk)
    t_near, m = _near(c, start, topk, kappa)
    z = np.zeros_like(c)
    for j in range(topk):
        w, _ = _weight(c, (start + j).astype(np.float32), t_near, m, kappa)
        z = (z + w).astype(np.float32)
    uz = (u * z).astype(np.float32)
    acc = np.zeros_like(c)
    cnt = np.zeros(c.shape, dtype=np.int64)
    for j in range(topk):
        w, _ = _weight(c, (start + j).astype(np.float32), t_near, m, kappa)
        acc = (acc + w).astype(np.float32)
        cnt += (acc <= uz)
    return start + np.minimum(cnt, topk - 1)


def probabilities(f: Format, v, kappa, topk):
    """P(level start + j) for each element: the sampler's distribution."""
    kappa = np.float32(kappa)
    c, start, _ = _window(f, v, topk)
    t_near, m = _near(c, start, topk, kappa)
    ws = np.stack([_weight(c, (start + j).astype(np.float32), t_near, m, kappa)[0] for j in range(topk)], -1)
    return start, ws / ws.sum(-1, keepdims=True)


def proxy_coeffs(f: Format, v, kappa, topk):
    kappa = np.float32(kappa)
    c, start, kgap = _window(f, v, topk)
    t_near, m = _near(c, start, topk, kappa)
    z = sl = sa = sal = sb = sbl = np.zeros_like(c)
    for j in range(topk):
        t = (start + j).astype(np.float32)
        e, d = _weight(c, t, t_near, m, kappa)
        lv = f.level[start + j]
        a = np.float32(-2.0) * kappa * d
        z = z + e
        sl = sl + e * lv
        sa = sa + e * a
        sal = sal + e * a * lv
        sb = sb + e * d * d
        sbl = sbl + e * d * d * lv
    p_lt = sl / z
    dth = (sal / z - p_lt * (sa / z)) / kgap
    ds = p_lt - v * dth
    dk = p_lt * (sb / z) - sbl / z
    return dth.astype(np.float32), ds.astype(np.float32), dk.astype(np.float32)


# ---------------------------------------------------------------------------
# forward / backward of one ECDL quantize
# ---------------------------------------------------------------------------
def _scales(f: Format, raw, mode):
    """(q indices [m, nb], s [m, nb], alpha) for theta [m, nb, tpb]."""
    bamax = np.abs(raw).max(-1).astype(np.float32)
    if mode == MODE_NVIDIA:
        gmax = np.maximum(bamax.max(), TINY).astype(np.float32)
        # torch divides a tensor by a Python float as a multiply by the fp32 reciprocal
        alpha = np.float32(gmax * np.float32(np.float32(1.0) / np.float32(f.f_max)))
        qv = ((bamax * f.q_max).astype(np.float32) / gmax).astype(np.float32)
        qi = f.q_ordinal(qv)
    else:
        alpha = np.float32(1.0)
        bits = np.maximum(bamax, TINY).view(np.uint32).astype(np.int64)
        qi = np.clip(((bits >> 23) - 127) - f.emax + 127, 0, 254)
    s = (f.q[qi] * alpha).astype(np.float32)
    return qi, s, alpha


def forward(fmt: int, theta: np.ndarray, kappa: float, seed: int, topk: int, mode: int):
    """theta: float32 [m, nb, tpb].  Returns (packed codes, scale bytes [m, nb],
    alpha, sampled level indices [m, nb, tpb])."""
    f = Format(fmt)
    m_, nb, tpb = theta.shape
    raw = theta.astype(np.float32)
    qi, s, alpha = _scales(f, raw, mode)
    v = (raw / s[..., None]).astype(np.float32)
    k = nb * tpb
    offs = (np.arange(m_)[:, None, None] * k + np.arange(nb)[None, :, None] * tpb
            + np.arange(tpb)[None, None, :]).astype(np.uint64)
    u = uniform(seed, offs)
    idx = sample(f, v, kappa, u, topk)
    if f.tn == 16:
        code = np.where(idx < 8, 15 - idx, idx - 8).astype(np.uint8)
        packed = (code[..., 0::2] | (code[..., 1::2] << 4)).astype(np.uint8).reshape(m_, nb * tpb // 2)
    else:
        packed = np.where(idx < 127, 254 - idx, idx - 127).astype(np.uint8).reshape(m_, nb * tpb)
    return packed, (qi + f.bias).astype(np.uint8), alpha, idx


def backward(fmt: int, g: np.ndarray, theta: np.ndarray, scale_bytes: np.ndarray, kappa: float, alpha: float,
             topk: int):
    """dtheta [m, nb, tpb] (float32) and the scalars (d kappa, d alpha)."""
    f = Format(fmt)
    qi = np.maximum(scale_bytes.astype(np.int64) - f.bias, 0)
    q_hat = f.q[qi]
    s = (q_hat * np.float32(alpha)).astype(np.float32)
    v = (theta.astype(np.float32) / s[..., None]).astype(np.float32)
    dth, ds_c, dk = proxy_coeffs(f, v, kappa, topk)
    g = g.astype(np.float32)
    dtheta = g * dth
    dkt = float(np.sum(g.astype(np.float64) * s[..., None] * dk))
    dal = float(np.sum(g.astype(np.float64) * ds_c * q_hat[..., None]))
    return dtheta.astype(np.float32), (dkt, dal)


# ---------------------------------------------------------------------------
# CCDL (cdl/core/kernel/ccdl/kernel.py, primitives.py:73-135 and 190-240):
# the block scale is itself a learnable value q, sampled on the scale levels
# with the truncated window; theta as in ECDL
# ---------------------------------------------------------------------------
class QFormat:
    """The scale format's levels as a sampling grid (UE4M3 without zero for
    NVFP4, E8M0 for MX)."""

    def __init__(self, fmt: int):
        self.fmt = fmt
        self.level = q_levels(fmt)
        self.gap = gaps(self.level)
        self.tn = self.level.size
        self.bias = 1 if fmt == NVFP4 else 0

    def ordinal(self, v):
        if self.fmt == NVFP4:
            b = e4m3_rne(np.clip(v, np.float32(2.0 ** -9), np.float32(448.0)))
            return np.clip(b - 1, 0, self.tn - 1)
        v = np.clip(np.asarray(v, np.float32), np.float32(2.0 ** -127), np.float32(2.0 ** 127)).astype(np.float32)
        bits = v.view(np.uint32).astype(np.int64)
        e8, mant = bits >> 23, bits & 0x7FFFFF
        return np.where(e8 == 0, (mant > 4194304).astype(np.int64), np.minimum(e8 + (mant >= 4194304), self.tn - 1))


def _half_window(topk, kappa):
    hq = topk // 2
    if kappa > 0.05:
        hq = int(min(float(topk // 2), float(np.sqrt(np.float32(60.0) / np.float32(kappa))))) + 1
    return hq


def sample_truncated(f, v, kappa, u, topk):
    kappa = np.float32(kappa)
    c, start, _ = _window(f, v, topk)
    t_near, m = _near(c, start, topk, kappa)
    hq = _half_window(topk, kappa)
    t_lo = np.maximum(start, t_near - hq)
    z = np.zeros_like(c)
    for j in range(2 * hq + 1):
        t = t_lo + j
        inw = (t >= start) & (t <= start + topk - 1)
        w, _ = _weight(c, t.astype(np.float32), t_near, m, kappa)
        z = (z + np.where(inw, w, np.float32(0.0))).astype(np.float32)
    d_left = ((t_lo - 1).astype(np.float32) - c).astype(np.float32)
    e_left = np.exp2((np.minimum((-kappa * d_left * d_left - m).astype(np.float32), np.float32(0.0))
                      * LOG2E).astype(np.float32)).astype(np.float32)
    uz = (u * z).astype(np.float32)
    off = np.where(uz >= (e_left * ((t_lo - start).astype(np.float32) + np.float32(1.0))).astype(np.float32),
                   t_lo - start, 0)
    acc = np.zeros_like(c)
    cnt = np.zeros(c.shape, dtype=np.int64)
    for j in range(2 * hq + 1):
        t = t_lo + j
        inw = (t >= start) & (t <= start + topk - 1)
        w, _ = _weight(c, t.astype(np.float32), t_near, m, kappa)
        acc = (acc + np.where(inw, w, np.float32(0.0))).astype(np.float32)
        cnt += (acc <= uz) & inw
    return start + np.minimum(off + cnt, topk - 1)


def proxy_coeffs_truncated(f, v, kappa, topk):
    kappa = np.float32(kappa)
    c, start, kgap = _window(f, v, topk)
    t_near, m = _near(c, start, topk, kappa)
    hq = _half_window(topk, kappa)
    t_lo = np.maximum(start, t_near - hq)
    z = sl = sa = sal = sb = sbl = np.zeros_like(c)
    for j in range(2 * hq + 1):
        t = t_lo + j
        inw = (t >= start) & (t <= start + topk - 1)
        e, d = _weight(c, t.astype(np.float32), t_near, m, kappa)
        lv = f.level[np.minimum(t, start + topk - 1)]
        a = np.float32(-2.0) * kappa * d
        w = np.where(inw, e, np.float32(0.0))
        z = z + w
        sl = sl + w * lv
        sa = sa + w * a
        sal = sal + w * a * lv
        sb = sb + w * d * d
        sbl = sbl + w * d * d * lv
    p_lt = sl / z
    dth = (sal / z - p_lt * (sa / z)) / kgap
    ds = p_lt - v * dth
    dk = p_lt * (sb / z) - sbl / z
    return dth.astype(np.float32), ds.astype(np.float32), dk.astype(np.float32)


def ccdl_forward(fmt: int, theta: np.ndarray, q: np.ndarray, kappa_t: float, kappa_q: float, alpha: float,
                 seed: int, topk: int, q_topk: int):
    """theta [m, nb, tpb], q [m, nb] or [1, nb] (shared).  Returns (packed
    codes, scale bytes [m, nb] (or [1, nb] when q is shared))."""
    f, fq = Format(fmt), QFormat(fmt)
    m_, nb, tpb = theta.shape
    k = nb * tpb
    qs = 0 if q.shape[0] == 1 and m_ > 1 else nb
    qq = np.broadcast_to(q.astype(np.float32), (m_, nb))
    uq_off = (m_ * k + np.arange(m_)[:, None] * qs + np.arange(nb)[None, :]).astype(np.uint64)
    uq = uniform(seed, uq_off)
    qi = sample_truncated(fq, qq, kappa_q, uq, q_topk)
    s = (fq.level[qi] * np.float32(alpha)).astype(np.float32)
    v = (theta.astype(np.float32) / s[..., None]).astype(np.float32)
    offs = (np.arange(m_)[:, None, None] * k + np.arange(nb)[None, :, None] * tpb
            + np.arange(tpb)[None, None, :]).astype(np.uint64)
    idx = sample(f, v, kappa_t, uniform(seed, offs), topk)
    if f.tn == 16:
        code = np.where(idx < 8, 15 - idx, idx - 8).astype(np.uint8)
        packed = (code[..., 0::2] | (code[..., 1::2] << 4)).astype(np.uint8).reshape(m_, nb * tpb // 2)
    else:
        packed = np.where(idx < 127, 254 - idx, idx - 127).astype(np.uint8).reshape(m_, nb * tpb)
    scale = (qi + fq.bias).astype(np.uint8)
    return packed, (scale[:1] if qs == 0 else scale)


def ccdl_backward(fmt: int, g, theta, q, scale_bytes, kappa_t, kappa_q, alpha, topk, q_topk):
    """(dtheta [m, nb, tpb], dq [m, nb] per theta row, (d kappa_t, d kappa_q, d alpha))."""
    f, fq = Format(fmt), QFormat(fmt)
    m_, nb, tpb = theta.shape
    sb = np.broadcast_to(scale_bytes, (m_, nb))
    qi = np.maximum(sb.astype(np.int64) - fq.bias, 0)
    q_hat = fq.level[qi]
    s = (q_hat * np.float32(alpha)).astype(np.float32)
    v = (theta.astype(np.float32) / s[..., None]).astype(np.float32)
    dth, ds_c, dk = proxy_coeffs(f, v, kappa_t, topk)
    g = g.astype(np.float32)
    ds = g * ds_c
    dkt = float(np.sum(g.astype(np.float64) * s[..., None] * dk))
    dal = float(np.sum(ds.astype(np.float64) * q_hat[..., None]))
    qq = np.broadcast_to(q.astype(np.float32), (m_, nb))
    dq_c, _, dkq_t = proxy_coeffs_truncated(fq, qq, kappa_q, q_topk)
    gq = (np.float32(alpha) * ds.sum(-1)).astype(np.float32)
    dq = (gq * dq_c).astype(np.float32)
    dkq = float(np.sum(gq.astype(np.float64) * dkq_t))
    return (g * dth).astype(np.float32), dq, (dkt, dkq, dal)


def _bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    return r.view(np.float32)


def ccdl_round(fmt: int, theta: np.ndarray, q: np.ndarray, alpha: float, theta_bf16: bool, levels_bf16: bool):
    """CCDL eval forward, ``cascaded_nearest_round`` (cdl/core/ccdl.py:78-89):
    ``q`` to its nearest scale level, ``s = level * alpha`` in the level dtype,
    theta to the nearest level of ``theta / s`` in the promoted dtype of theta
    and the levels (a bf16 tensor times or over a bf16 or 0-d fp32 tensor is
    computed in fp32 and rounded once to bf16).  theta [m, nb, tpb] (values
    already representable in its dtype), q [m, nb] or [1, nb].  Returns
    (packed codes, scale bytes shaped like q)."""
    f, fq = Format(fmt), QFormat(fmt)
    m_, nb, tpb = theta.shape
    qi = fq.ordinal(np.asarray(q, np.float32))
    s = (fq.level[qi] * np.float32(alpha)).astype(np.float32)
    if levels_bf16:
        s = _bf16(s)
    qb = np.broadcast_to(s, (m_, nb))
    v = (theta.astype(np.float32) / qb[..., None]).astype(np.float32)
    if levels_bf16 and theta_bf16:
        v = _bf16(v)
    idx = f.ordinal(v)
    if f.tn == 16:
        code = np.where(idx < 8, 15 - idx, idx - 8).astype(np.uint8)
        packed = (code[..., 0::2] | (code[..., 1::2] << 4)).astype(np.uint8).reshape(m_, nb * tpb // 2)
    else:
        packed = np.where(idx < 127, 254 - idx, idx - 127).astype(np.uint8).reshape(m_, nb * tpb)
    return packed, (qi + fq.bias).astype(np.uint8)
