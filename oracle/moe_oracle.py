"""CPU oracle for the sparse-MoE layer (test infrastructure, not product code).

This module is the parity checker for the CUDA path. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it. The product path (``phantom_moe``) never calls into it.

It restates, in NumPy, the reference's MoE-layer arithmetic:

* router: logits = x . Wr^T, softmax in fp32, top-k, renormalise
  (reference: tests/test_moe_routing.py:56-72 ``PhantomTopKRouter.forward``;
  executed form transformers 5.5.0 models/qwen3_moe/modeling_qwen3_moe.py:263-272
  ``Qwen3MoeTopKRouter.forward``; Mixtral models/mixtral/modeling_mixtral.py:109-117);
* dispatch: one_hot + where grouping of (token, slot) pairs per expert
  (modeling_qwen3_moe.py:234-244);
* expert SwiGLU FFN: gate = first half of ``gate_up_proj``, silu(gate) * up,
  then ``down_proj`` (modeling_qwen3_moe.py:245-247);
* combine: multiply by the routing weight and ``index_add_`` per token
  (modeling_qwen3_moe.py:248-249);
* int4 dequant: GGUF Q4_0 nibble order and the -8 offset
  (python/phantom/loader/gguf_loader.py:362-381 on CPU, 588-596 on GPU).

Two router forms live here. ``route_reference`` is the plain fp32 semantics
(what transformers computes, up to summation order). ``route_fixed_order``
replays, operation by operation, the fixed reduction order and the exp
routine of the CUDA router, so its logits, probabilities and top-k indices
are bit-identical to the kernel's. Both are pinned against the reference: the
golden fixtures under ``tests/golden`` were produced by running transformers'
``Qwen3MoeSparseMoeBlock`` / ``MixtralSparseMoeBlock``, the reference's own
``PhantomTopKRouter`` and the reference's ``GGUFLoader.dequantize_tensor``.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# int4 symmetric group quantisation (build-defined format)
# ---------------------------------------------------------------------------
#
# Layout of one row of K weights, group size G (32 or 64), K % G == 0:
#   value = (nibble - 8) * scale, one fp16 scale per G consecutive elements in
#   a separate [rows, K/G] array (GGUF Q4_0 semantics, gguf_loader.py:362-381,
#   with the block's fp16 `d` moved out and the group generalised to 64).
#   Nibble order (build-defined, chosen for the GPU dequantiser): every 8
#   consecutive elements e0..e7 form one little-endian 32-bit word with
#   element e_{2i} in bits [4i, 4i+4) and e_{2i+1} in bits [16+4i, 16+4i+4),
#   i = 0..3; i.e. bytes (e0|e2<<4, e4|e6<<4, e1|e3<<4, e5|e7<<4). Shifting the
#   word right by 4i and masking 0x000F000F yields the pair (e_{2i}, e_{2i+1})
#   in the two 16-bit halves - one bf16x2 register per instruction.
#   GGUF Q4_0 blocks convert to this layout losslessly (a nibble shuffle,
#   :func:`q4_0_to_packed`).
# Quantiser (the reference has none; it consumes GGUF files):
#   scale = fp16(absmax(group) / 7), q = clamp(rint(w / scale), -8, 7).

# element (within its 8-element word) held by the low / high nibble of byte p
_LO_ELEM = np.array([0, 4, 1, 5])
_HI_ELEM = _LO_ELEM + 2


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """Nibble values ``q[..., K]`` (0..15, K % 8 == 0) -> packed ``[..., K/2]``."""
    q = np.asarray(q, dtype=np.uint8)
    lead, K = q.shape[:-1], q.shape[-1]
    qw = q.reshape(*lead, K // 8, 8)
    packed = qw[..., _LO_ELEM] | (qw[..., _HI_ELEM] << 4)
    return packed.astype(np.uint8).reshape(*lead, K // 2)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_nibbles`: ``[..., K/2]`` -> nibble values ``[..., K]``."""
    packed = np.asarray(packed, dtype=np.uint8)
    lead, K = packed.shape[:-1], packed.shape[-1] * 2
    pw = packed.reshape(*lead, K // 8, 4)
    q = np.empty((*lead, K // 8, 8), dtype=np.uint8)
    q[..., _LO_ELEM] = pw & 0x0F
    q[..., _HI_ELEM] = pw >> 4
    return q.reshape(*lead, K)


def quantize_int4(w: np.ndarray, group: int = 64):
    """Quantise ``w[..., K]`` (fp32) to packed int4 + fp16 scales.

    Returns ``(packed uint8[..., K/2], scales fp16[..., K/group])``.
    """
    w = np.ascontiguousarray(w, dtype=F32)
    K = w.shape[-1]
    assert K % group == 0 and group in (32, 64)
    lead = w.shape[:-1]
    wg = w.reshape(*lead, K // group, group)
    absmax = np.max(np.abs(wg), axis=-1)
    scale16 = (absmax / F32(7.0)).astype(np.float16)
    s = scale16.astype(F32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s > 0, np.rint(wg / np.where(s > 0, s, F32(1.0))), F32(0.0))
    q = (np.clip(q, -8, 7).astype(np.int16) + 8).astype(np.uint8).reshape(*lead, K)
    return pack_nibbles(q), scale16


def dequantize_int4(packed: np.ndarray, scales: np.ndarray, group: int = 64) -> np.ndarray:
    """Inverse of :func:`quantize_int4` (fp32 output): (nibble - 8) * scale,
    as gguf_loader.py:372-378 dequantises Q4_0 with a per-block ``d``."""
    q = unpack_nibbles(packed).astype(np.int16) - 8
    lead, K = q.shape[:-1], q.shape[-1]
    s = scales.astype(F32)[..., None]
    return (q.reshape(*lead, K // group, group).astype(F32) * s).reshape(*lead, K)


def dequantize_q4_0(raw: bytes, n_elems: int) -> np.ndarray:
    """GGUF Q4_0 blocks -> fp32 (restates gguf_loader.py:362-381).

    The reference returns bf16 (gguf_loader.py:380); this returns the fp32
    values before that rounding.
    """
    n_blocks = n_elems // 32
    blk = np.frombuffer(raw[: n_blocks * 18], dtype=np.uint8).reshape(n_blocks, 18)
    d = blk[:, :2].copy().view(np.float16).astype(F32)
    qs = blk[:, 2:]
    low = (qs & 0x0F).astype(np.int8) - 8
    high = ((qs >> 4) & 0x0F).astype(np.int8) - 8
    out = np.empty((n_blocks, 32), dtype=F32)
    out[:, :16] = low * d
    out[:, 16:] = high * d
    return out.reshape(-1)[:n_elems]


def q4_0_to_packed(raw: bytes, rows: int, K: int):
    """Convert GGUF Q4_0 blocks of a [rows, K] tensor into (packed, scales).

    Lossless: each 18-byte block's fp16 ``d`` goes to the scales array (group
    size 32) and its 32 nibbles (byte j: element j low, element j+16 high,
    gguf_loader.py:372-378) are re-ordered into the packed nibble layout.
    """
    nb = K // 32
    blk = np.frombuffer(raw[: rows * nb * 18], dtype=np.uint8).reshape(rows, nb, 18)
    scales = blk[:, :, :2].copy().view(np.float16).reshape(rows, nb)
    qs = blk[:, :, 2:]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=-1).reshape(rows, K)
    return pack_nibbles(q), scales


def dequantize_q4_k(raw: bytes, n_elems: int) -> np.ndarray:
    """GGUF Q4_K super-blocks -> fp32 (restates ``dequantize_tensor_cuda``,
    gguf_loader.py:648-666, the dequantiser the reference's model loader runs
    at gguf_loader.py:799; that function's fp32 values before the bf16 cast).

    Super-block of 256 elements, 144 bytes: fp16 d, fp16 dmin, 12 bytes of
    packed 6-bit (scale, min) pairs for 8 sub-blocks of 32, 128 bytes of
    nibbles; 32-byte chunk c holds sub-block 2c in its low and 2c+1 in its
    high nibbles. value = fp32(d * sc_j) * q - fp32(dmin * m_j), each product
    and the difference rounded to fp32. (The reference's CPU branch,
    gguf_loader.py:453-489, orders the nibbles differently; the loader does
    not use it for this path.)
    """
    nb = n_elems // 256
    blk = np.frombuffer(raw[: nb * 144], dtype=np.uint8).reshape(nb, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(F32)       # [nb, 1]
    dmin = blk[:, 2:4].copy().view(np.float16).astype(F32)
    s = blk[:, 4:16].astype(np.int32)
    sc = np.concatenate([s[:, 0:4] & 0x3F, (s[:, 8:12] & 0x0F) | ((s[:, 0:4] >> 6) << 4)], axis=1)
    mn = np.concatenate([s[:, 4:8] & 0x3F, (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)], axis=1)
    d_sc = (d * sc.astype(F32)).astype(F32)[:, :, None]       # [nb, 8, 1]
    dm_m = (dmin * mn.astype(F32)).astype(F32)[:, :, None]
    qs = blk[:, 16:].reshape(nb, 4, 1, 32)
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=2).reshape(nb, 8, 32).astype(F32)
    return ((d_sc * q).astype(F32) - dm_m).astype(F32).reshape(-1)[:n_elems]


def q4_k_to_packed(raw: bytes, rows: int, K: int, group: int = 32):
    """Import a GGUF Q4_K [rows, K] tensor into (packed, scales): dequantise
    as :func:`dequantize_q4_k`, then re-quantise with :func:`quantize_int4`
    (the symmetric format cannot hold Q4_K's per-sub-block minimum, so this
    import is lossy, unlike :func:`q4_0_to_packed`)."""
    w = dequantize_q4_k(raw, rows * K).reshape(rows, K)
    return quantize_int4(w, group)


# ---------------------------------------------------------------------------
# fixed-order fp32 arithmetic shared with the CUDA router
# ---------------------------------------------------------------------------

def _bits(u: int) -> np.float32:
    return np.array(u, dtype=np.uint32).view(F32)[()]


# Constants as exact fp32 bit patterns (the CUDA router uses the same bits).
LOG2E = _bits(0x3FB8AA3B)   # log2(e)
LN2_HI = _bits(0x3F318000)  # 0.693359375, 9 significant bits: n * LN2_HI is exact
LN2_LO = _bits(0xB95E8083)  # ln(2) - LN2_HI
EXP_C = [_bits(u) for u in (0x3F800000, 0x3F800000, 0x3F000000, 0x3E2AAAAB,
                            0x3D2AAAAB, 0x3C088889, 0x3AB60B61, 0x39500D01)]  # 1/i!


def fixed_exp(x: np.ndarray) -> np.ndarray:
    """exp(x) for x <= 0 by Cody-Waite range reduction + degree-7 Taylor.

    Every step is one correctly rounded fp32 operation (no fused multiply-add),
    in the same order as ``phm_exp_fixed`` in the CUDA router, so both produce
    identical bits. x < -87 returns 0.
    """
    x = np.asarray(x, dtype=F32)
    n = np.rint((x * LOG2E).astype(F32)).astype(F32)
    r = (x - (n * LN2_HI).astype(F32)).astype(F32)
    r = (r - (n * LN2_LO).astype(F32)).astype(F32)
    p = EXP_C[7]
    for c in (EXP_C[6], EXP_C[5], EXP_C[4], EXP_C[3], EXP_C[2], EXP_C[1], EXP_C[0]):
        p = ((p * r).astype(F32) + c).astype(F32)
    ni = np.clip(n, -126, 127).astype(np.int32)
    two_n = ((ni + 127).astype(np.uint32) << np.uint32(23)).view(F32)
    out = (p * two_n).astype(F32)
    return np.where(x < F32(-87.0), F32(0.0), out).astype(F32)


LANES = 32
VEC = 8  # elements per lane per chunk (one 16-byte load of bf16)


def logits_fixed_order(x: np.ndarray, wr: np.ndarray, products_exact: bool) -> np.ndarray:
    """Router logits in the CUDA router's reduction order.

    Element h of the hidden dimension goes to lane (h // 8) % 32 of a warp;
    each lane accumulates its elements in increasing h with a rounded multiply
    then a rounded add; the 32 lane sums are combined by an xor butterfly
    (offsets 16, 8, 4, 2, 1). H is zero-padded to a multiple of 256.
    ``products_exact`` is informational (bf16 inputs give exact fp32
    products); the arithmetic is identical either way.
    """
    x = np.asarray(x, dtype=F32)
    wr = np.asarray(wr, dtype=F32)
    T, H = x.shape
    E = wr.shape[0]
    Hp = ((H + LANES * VEC - 1) // (LANES * VEC)) * LANES * VEC
    if Hp != H:
        x = np.pad(x, ((0, 0), (0, Hp - H)))
        wr = np.pad(wr, ((0, 0), (0, Hp - H)))
    nchunk = Hp // (LANES * VEC)
    xr = x.reshape(T, nchunk, LANES, VEC)
    wrr = wr.reshape(E, nchunk, LANES, VEC)
    acc = np.zeros((T, E, LANES), dtype=F32)
    for c in range(nchunk):
        for v in range(VEC):
            prod = (xr[:, None, c, :, v] * wrr[None, :, c, :, v]).astype(F32)
            acc = (acc + prod).astype(F32)
    for off in (16, 8, 4, 2, 1):
        perm = np.arange(LANES) ^ off
        acc = (acc + acc[:, :, perm]).astype(F32)
    return acc[:, :, 0].copy()


def softmax_fixed(logits: np.ndarray) -> np.ndarray:
    """Softmax in the CUDA router's order: max, exp(l - max), lane sums
    (expert e on lane e % 32, ascending e), xor butterfly, then a rounded
    division."""
    l = np.asarray(logits, dtype=F32)
    T, E = l.shape
    m = l.max(axis=1, keepdims=True)
    e = fixed_exp((l - m).astype(F32))
    Ep = ((E + LANES - 1) // LANES) * LANES
    ep = np.pad(e, ((0, 0), (0, Ep - E))).reshape(T, Ep // LANES, LANES)
    acc = np.zeros((T, LANES), dtype=F32)
    for i in range(Ep // LANES):
        acc = (acc + ep[:, i, :]).astype(F32)
    for off in (16, 8, 4, 2, 1):
        perm = np.arange(LANES) ^ off
        acc = (acc + acc[:, perm]).astype(F32)
    s = acc[:, :1]
    return (e / s).astype(F32)


def topk_stable(p: np.ndarray, k: int):
    """Top-k by descending value; equal values -> lower expert index first.

    The reference uses ``torch.topk`` whose tie order is unspecified
    (modeling_qwen3_moe.py:267); this build pins 'lower index wins'.
    """
    T, E = p.shape
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -p), axis=1)[:, :k]
    return order.astype(np.int32), np.take_along_axis(p, order, axis=1).astype(F32)


def renormalise_fixed(vals: np.ndarray, renormalize: bool) -> np.ndarray:
    """Sum of the k picked probabilities in pick order, then divide
    (modeling_qwen3_moe.py:268-269)."""
    if not renormalize:
        return vals.astype(F32)
    s = np.zeros((vals.shape[0], 1), dtype=F32)
    for j in range(vals.shape[1]):
        s = (s + vals[:, j : j + 1]).astype(F32)
    return (vals / s).astype(F32)


def route_fixed_order(x, wr, top_k: int, renormalize: bool = True):
    """Router exactly as the CUDA kernel computes it.

    Returns (logits fp32[T,E], probs fp32[T,E], idx int32[T,k], w fp32[T,k]).
    """
    logits = logits_fixed_order(x, wr, products_exact=True)
    probs = softmax_fixed(logits)
    idx, vals = topk_stable(probs, top_k)
    return logits, probs, idx, renormalise_fixed(vals, renormalize)


def sigmoid_fixed(x: np.ndarray) -> np.ndarray:
    """sigmoid as the CUDA router computes it: 1 / (1 + exp(-x)) for x >= 0,
    e / (1 + e) with e = exp(x) otherwise, exp by :func:`fixed_exp`, each
    step rounded to fp32."""
    x = np.asarray(x, dtype=F32)
    pos = x >= 0
    e = fixed_exp(np.where(pos, -x, x).astype(F32))
    den = (F32(1.0) + e).astype(F32)
    return np.where(pos, (F32(1.0) / den).astype(F32), (e / den).astype(F32)).astype(F32)


def route_sigmoid_grouped(x, wr, top_k: int, renormalize: bool = True, score_bias=None, n_group: int = 1,
                          topk_group: int = 1, routed_scale: float = 1.0, logits=None):
    """DeepSeek-V3 routing (transformers 5.5.0 models/deepseek_v3/modeling_deepseek_v3.py
    DeepseekV3MoE.route_tokens_to_experts) as the CUDA router computes it:
    s = sigmoid(logits); choice c = s + bias; groups of E/n_group score the
    sum of their two largest c; the topk_group best groups stay, the rest
    get c = 0; top_k largest c (ties -> lower index; the reference's
    ``topk(sorted=False)`` leaves the order open); weights = s of the picks,
    over (their sum in pick order + 1e-20) when renormalising, times
    routed_scale. Returns (logits, s, idx, w)."""
    if logits is None:
        logits = logits_fixed_order(x, wr, products_exact=True)
    logits = np.asarray(logits, dtype=F32)
    s = sigmoid_fixed(logits)
    c = (s + np.asarray(score_bias, dtype=F32)).astype(F32) if score_bias is not None else s.copy()
    T, E = c.shape
    if n_group > 1:
        gs = E // n_group
        top2 = -np.sort(-c.reshape(T, n_group, gs), axis=2)[:, :, :2]
        gscore = (top2[:, :, 0] + top2[:, :, 1]).astype(F32)
        gsel = np.argsort(-gscore, axis=1, kind="stable")[:, :topk_group]
        keep = np.zeros((T, n_group), dtype=bool)
        np.put_along_axis(keep, gsel, True, axis=1)
        c = np.where(np.repeat(keep, gs, axis=1), c, F32(0.0)).astype(F32)
    idx = np.argsort(-c, axis=1, kind="stable")[:, :top_k].astype(np.int32)
    w = np.take_along_axis(s, idx, axis=1).astype(F32)
    if renormalize:
        tot = np.zeros(T, dtype=F32)
        for j in range(top_k):
            tot = (tot + w[:, j]).astype(F32)
        w = (w / (tot + F32(1e-20)).astype(F32)[:, None]).astype(F32)
    return logits, s, idx, (w * F32(routed_scale)).astype(F32)


def route_reference(x, wr, top_k: int, renormalize: bool = True):
    """Plain fp32 router semantics (modeling_qwen3_moe.py:263-272): logits by
    float64 dot then rounded to fp32, fp32 softmax, stable top-k, renorm."""
    x = np.asarray(x, dtype=np.float64)
    wr = np.asarray(wr, dtype=np.float64)
    logits = (x @ wr.T).astype(F32)
    l64 = logits.astype(np.float64)
    e = np.exp(l64 - l64.max(axis=1, keepdims=True))
    probs = (e / e.sum(axis=1, keepdims=True)).astype(F32)
    idx, vals = topk_stable(probs, top_k)
    if renormalize:
        vals = (vals / vals.sum(axis=1, keepdims=True, dtype=np.float64)).astype(F32)
    return logits, probs, idx, vals


def topk_margin(probs: np.ndarray, k: int) -> np.ndarray:
    """Per-token gap between the k-th and (k+1)-th largest probability."""
    s = -np.sort(-probs, axis=1)
    if probs.shape[1] <= k:
        return np.full(probs.shape[0], np.inf, dtype=F32)
    return (s[:, k - 1] - s[:, k]).astype(F32)


# ---------------------------------------------------------------------------
# fixed-point rows: the operand format of the decode FFN
# ---------------------------------------------------------------------------
#
# The CUDA decode FFN multiplies the int4 nibbles with activations and SwiGLU
# outputs held as exact integers (build-defined; the reference multiplies in
# fp32, modeling_qwen3_moe.py:245-247, on weights dequantised as
# (nibble - 8) * scale, gguf_loader.py:372-378):
#   per row and group of G elements, e = the exponent that scales the group's
#   largest |value| m into [2^12, 8191] (G = 64) or [2^13, 16383] (G = 32),
#   clamped to [-126, 100]; A = rint(v * 2^-e), |A| <= 8191 (16383);
#   A = 256 * hi + lo with hi = (A + 128) >> 8 and lo = A - 256 * hi, both
#   signed bytes; bytes of each 8-element word: the 8 high bytes then the 8
#   low bytes (two's complement; the low byte is A & 255), each in element
#   order 0, 4, 1, 5, 2, 6, 3, 7;
#   constants {C0, M}: M = the int32 bits of the float 1.5 * 2^(23 + e),
#   C0 = M - 8 * sum(A).
# For nibbles n the group sum v = sum((n - 8) * A) is an exact integer with
# |v| < 2^22, so the int32 M + v, read as a float, minus the float of M is
# v * 2^e with no rounding (fx_group_dot replays this).

FX_MAGIC = 0x4B400000
FX_MIN_EXP, FX_MAX_EXP = -126, 100
_FX_SLOT_ELEM = np.array([0, 4, 1, 5, 2, 6, 3, 7])  # element held by byte slot j of a plane


def fx_limits(group: int):
    """(amax, shift, limit) of the fixed-point groups of size ``group``."""
    return (8191, 12, 8191.5) if group == 64 else (16383, 13, 16383.5)


def fx_exponents(v: np.ndarray, group: int):
    """Per-group exponents of ``v [..., K]`` (fp32 values) and a flag per
    group that holds a value it cannot represent (beyond the range, infinite
    or NaN; the kernels raise device error bit value 2 for it). As in the
    kernels, the group maximum ignores NaNs (fmaxf) and a maximum above
    3e38 takes the largest exponent."""
    _, shift, lim = fx_limits(group)
    v = np.asarray(v, dtype=F32)
    vg = np.abs(v.reshape(*v.shape[:-1], v.shape[-1] // group, group).astype(np.float64))
    big = float(F32(3.0e38))
    with np.errstate(invalid="ignore"):
        flag = ~np.all(vg <= big, axis=-1)
        m = np.where(np.isnan(vg), 0.0, vg).max(axis=-1)
        top = ~(m <= big)
        _, p = np.frexp(np.where(top, 1.0, m))  # m = f * 2^p, f in [0.5, 1): floor(log2 m) = p - 1
    e0 = (p - 1 - shift).astype(np.int64)
    e = np.where(m * np.exp2(-e0.astype(np.float64)) >= lim, e0 + 1, e0)
    e = np.where(e0 < FX_MIN_EXP, FX_MIN_EXP, e)   # tiny groups: the smallest exponent, no rounding up
    e = np.where(m == 0, 0, e)
    over = e > FX_MAX_EXP
    e = np.where(top | over, FX_MAX_EXP, e)
    return e, flag | over


def fx_encode_rows(v: np.ndarray, group: int):
    """Fixed-point rows of ``v [rows, K]`` (fp32): returns ``(A int32 [rows,
    K], e int64 [rows, K/G], q uint8 [rows, 2K], consts int32 [rows, K/G, 2],
    bad bool [rows, K/G])`` with the byte layout and constants the CUDA
    encoder writes (``phmoe_fx_rows``)."""
    amax, _, _ = fx_limits(group)
    v = np.asarray(v, dtype=F32)
    rows, K = v.shape
    e, bad = fx_exponents(v, group)
    scaled = v.astype(np.float64).reshape(rows, K // group, group) * np.exp2(-e.astype(np.float64))[..., None]
    with np.errstate(invalid="ignore"):
        a = np.where(np.isnan(scaled), 0.0, np.clip(np.rint(scaled), -amax, amax))
    A = a.astype(np.int64).reshape(rows, K)
    hi = (((A + 128) >> 8) & 255).astype(np.uint8).reshape(rows, K // 8, 8)[..., _FX_SLOT_ELEM]
    lo = (A & 255).astype(np.uint8).reshape(rows, K // 8, 8)[..., _FX_SLOT_ELEM]
    q = np.concatenate([hi, lo], axis=-1).reshape(rows, 2 * K)
    M = FX_MAGIC + e * (1 << 23)
    S = A.reshape(rows, K // group, group).sum(-1)
    consts = np.stack([M - 8 * S, M], axis=-1).astype(np.int32)
    return A.astype(np.int32), e, q, consts, bad


def fx_decode_q(q: np.ndarray) -> np.ndarray:
    """The integers A of fixed-point row bytes ``q [rows, 2K]``."""
    rows, K2 = q.shape
    w = q.reshape(rows, K2 // 16, 2, 8)
    hi = w[:, :, 0, :].astype(np.int8).astype(np.int64)
    lo = w[:, :, 1, :].astype(np.int8).astype(np.int64)
    A = np.empty((rows, K2 // 16, 8), dtype=np.int64)
    A[..., _FX_SLOT_ELEM] = hi * 256 + lo
    return A.reshape(rows, K2 // 2)


def fx_group_dot(nibbles: np.ndarray, A: np.ndarray, consts: np.ndarray) -> np.ndarray:
    """One group's dot product the way the tensor-core kernels form it:
    i_lo = C0 + sum(n * lo), i_hi = sum(n * hi) (exact int32; hi = (A + 128)
    >> 8 and lo = A - 256 * hi, both signed bytes), i = 256 * i_hi
    + i_lo, then float32(bits i) - float32(bits M). ``nibbles [G]`` (0..15),
    ``A [..., G]``, ``consts [..., 2]``; returns fp32 ``[...]`` equal to
    sum((n - 8) * A) * 2^e."""
    n = np.asarray(nibbles, dtype=np.int64)
    A = np.asarray(A, dtype=np.int64)
    hi = (A + 128) >> 8
    lo = A - 256 * hi
    i = 256 * (hi * n).sum(-1) + consts[..., 0].astype(np.int64) + (lo * n).sum(-1)
    assert np.all((i >= 0) & (i < 2 ** 31)), "int32 range"
    f = i.astype(np.uint32).view(F32)
    m = consts[..., 1].astype(np.uint32).view(F32)
    return (f - m).astype(F32)


# ---------------------------------------------------------------------------
# dispatch / FFN / combine
# ---------------------------------------------------------------------------


def dispatch(idx: np.ndarray, num_experts: int):
    """Group (token, slot) assignments by expert, ordered by token index.

    Returns ``counts[E]``, ``offsets[E+1]`` (exclusive scan), ``row_token[R]``
    (token of each permuted row), ``row_slot[R]`` (its k slot) and
    ``inv[T,k]`` (permuted row of each assignment); R = T*k.

    The reference groups with one_hot + where (modeling_qwen3_moe.py:234-244);
    within one expert each token appears at most once, so 'by token index' is
    a total order. This is the permutation the CUDA dispatch must reproduce
    bit for bit.
    """
    idx = np.asarray(idx, dtype=np.int64)
    T, k = idx.shape
    flat = idx.reshape(-1)
    # an expert id outside [0, E) is dropped, as the CUDA dispatch drops it:
    # no row, inverse -1 (R = the valid assignments)
    valid = (flat >= 0) & (flat < num_experts)
    a = np.nonzero(valid)[0]
    counts = np.bincount(flat[a], minlength=num_experts).astype(np.int32)
    offsets = np.zeros(num_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    tok = np.repeat(np.arange(T), k)[a]
    slot = np.tile(np.arange(k), T)[a]
    order = np.lexsort((tok, flat[a]))  # by expert, then token
    row_token = tok[order].astype(np.int32)
    row_slot = slot[order].astype(np.int32)
    inv = np.full(T * k, -1, dtype=np.int32)
    inv[a[order]] = np.arange(a.size, dtype=np.int32)
    return counts, offsets, row_token, row_slot, inv.reshape(T, k)


def silu(x):
    x = np.asarray(x, dtype=F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def expert_ffn(x_rows: np.ndarray, w13: np.ndarray, w2: np.ndarray) -> np.ndarray:
    """SwiGLU FFN of one expert in fp32 (modeling_qwen3_moe.py:245-247).

    ``w13`` is [2I, H] with the gate rows first (``chunk(2)`` order);
    ``w2`` is [H, I].
    """
    I = w13.shape[0] // 2
    gu = x_rows.astype(F32) @ w13.T.astype(F32)
    h = silu(gu[:, :I]) * gu[:, I:]
    return (h.astype(F32) @ w2.T.astype(F32)).astype(F32)


def moe_layer_reference(x, wr, w13_deq, w2_deq, top_k: int, renormalize: bool = True,
                        router: str = "fixed"):
    """Whole layer in fp32 on dequantized weights.

    ``router='fixed'`` uses the kernel-order router (so the expert choice is the
    kernel's), ``'reference'`` the plain fp32 router. Experts are visited in
    ascending index and their rows accumulated into each token in that order,
    as ``index_add_`` does (modeling_qwen3_moe.py:239-249).
    Returns (out fp32[T,H], idx, w).
    """
    x = np.asarray(x, dtype=F32)
    T, H = x.shape
    E = w13_deq.shape[0]
    if router == "fixed":
        _, _, idx, w = route_fixed_order(x, wr, top_k, renormalize)
    else:
        _, _, idx, w = route_reference(x, wr, top_k, renormalize)
    out = np.zeros((T, H), dtype=F32)
    for e in range(E):
        tok, slot = np.nonzero(idx == e)
        if tok.size == 0:
            continue
        y = expert_ffn(x[tok], w13_deq[e], w2_deq[e])
        out[tok] += (y * w[tok, slot][:, None]).astype(F32)
    return out, idx, w


def moe_layer_reference_packed(x, wr, w13_q, w13_s, w2_q, w2_s, top_k: int, group: int = 64,
                               renormalize: bool = True, router: str = "fixed", idx=None, w=None):
    """:func:`moe_layer_reference` on packed weights, dequantising one expert
    at a time (full-size layers would need ~2.4 GB of fp32 weights at once).
    ``idx``/``w`` may be given to reuse a routing computed elsewhere."""
    x = np.asarray(x, dtype=F32)
    T, H = x.shape
    E = w13_q.shape[0]
    if idx is None:
        route = route_fixed_order if router == "fixed" else route_reference
        _, _, idx, w = route(x, wr, top_k, renormalize)
    out = np.zeros((T, H), dtype=F32)
    for e in range(E):
        tok, slot = np.nonzero(idx == e)
        if tok.size == 0:
            continue
        d13 = dequantize_int4(w13_q[e], w13_s[e], group)
        d2 = dequantize_int4(w2_q[e], w2_s[e], group)
        y = expert_ffn(x[tok], d13, d2)
        out[tok] += (y * w[tok, slot][:, None]).astype(F32)
    return out, idx, w


def moe_layer_reference_shared(x, wr, w13_q, w13_s, w2_q, w2_s, top_k: int, num_shared: int, group: int = 64,
                               renormalize: bool = True, shared_gate=None, routed_scale: float = 1.0,
                               router: str = "fixed", scoring: str = "softmax", score_bias=None,
                               n_group: int = 1, topk_group: int = 1):
    """MoE block with shared experts on packed weights (experts E..E+m-1 are
    the m slices of the shared expert): routed output with weights times
    ``routed_scale``, plus g(t) * shared(x), g = sigmoid(x . shared_gate)
    (1 when None). Restates Qwen2MoeSparseMoeBlock.forward (transformers
    5.5.0 models/qwen2_moe/modeling_qwen2_moe.py: shared_expert_output scaled
    by F.sigmoid(shared_expert_gate(x)) and added to the routed output);
    DeepSeek blocks are the ungated case, routed by
    :func:`route_sigmoid_grouped` when ``scoring="sigmoid"``. Returns
    (out, routed idx, routed w before routed_scale)."""
    x = np.asarray(x, dtype=F32)
    T = x.shape[0]
    if scoring == "sigmoid":
        _, _, idx, w = route_sigmoid_grouped(x, wr, top_k, renormalize, score_bias, n_group, topk_group)
    else:
        route = route_fixed_order if router == "fixed" else route_reference
        _, _, idx, w = route(x, wr, top_k, renormalize)
    E = wr.shape[0]
    if shared_gate is None:
        g = np.ones((T, 1), dtype=F32)
    else:
        z = (x.astype(np.float64) @ np.asarray(shared_gate, dtype=np.float64).reshape(-1, 1))
        g = (1.0 / (1.0 + np.exp(-z))).astype(F32)
    idx2 = np.concatenate([idx, np.broadcast_to(E + np.arange(num_shared, dtype=idx.dtype), (T, num_shared))], 1)
    w2 = np.concatenate([(w * F32(routed_scale)).astype(F32), np.repeat(g, num_shared, axis=1)], 1)
    out, _, _ = moe_layer_reference_packed(x, wr, w13_q, w13_s, w2_q, w2_s, top_k + num_shared, group,
                                           idx=idx2, w=w2)
    return out, idx, w


def parity_stats(got: np.ndarray, ref: np.ndarray):
    """(max-abs error, mean-relative error) as the north star defines them:
    max |got - ref| and mean|got - ref| / mean|ref|."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got - ref)
    return float(d.max(initial=0.0)), float(d.mean() / max(np.abs(ref).mean(), 1e-30))


MAX_ABS_TOL = 2e-2
MEAN_REL_TOL = 5e-3
# Tighter bound the decode path meets on fp32 inputs (below the contract's
# MEAN_REL_TOL): its fixed-point operands hold every activation and SwiGLU
# value to 2^-13 of its group's largest |value|, which leaves ~3e-4 mean
# relative error against an fp32 computation.
DECODE_FP32_MEAN_REL = 1e-3
