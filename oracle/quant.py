"""Numpy restatement of the frozen-expert weight formats (test infrastructure).

Follows ``mirai/core/models/compressed_weights/quantization/quant.py`` of the
reference:

* INT8: ``_quantize_weight`` (quant.py:189-235) / ``_dequantize_weight``
  (quant.py:238-260) with the block-Hadamard rotation ``_hadamard``
  (quant.py:103-122) and ``best_group_size`` (quant.py:87-91).
* NF4: the reference calls bitsandbytes 0.49.2 ``quantize_4bit(bf16,
  blocksize=64, compress_statistics=True, quant_type="nf4")`` (quant.py:315-358)
  and dequantizes with ``dequantize_blockwise`` + ``dequantize_4bit``
  (quant.py:380-472).  bitsandbytes is not part of the reference tree, so this
  module restates the published methods:
    - the 4-bit NormalFloat table of QLoRA (Dettmers et al., 2023, sec. 3):
      quantiles of N(0,1) over 2^(k-1) negative and 2^(k-1)+1 positive ranges,
      one zero shared, normalised to [-1, 1];
    - blockwise absmax quantisation over 64 consecutive elements of the
      row-major flattened weight, two codes per byte, first element in the high
      nibble;
    - double quantisation of the fp32 absmax vector: subtract its mean
      (``offset``), then 8-bit blockwise quantisation (block 256) with the
      signed dynamic-tree map of "8-bit Optimizers via Block-wise
      Quantization" (Dettmers et al., 2022).
  Dequant is ``bf16(code[nibble] * (ncode[q] * nabsmax + offset))`` with each
  product and sum rounded in fp32, the order the reference pins in
  ``nf4_dequantize_stack`` (quant.py:413-431).
"""

from __future__ import annotations

import math

import numpy as np

NF4_BLOCKSIZE = 64
NF4_NESTED_BLOCKSIZE = 256
DEFAULT_GROUP_SIZES = (256, 64, 16)


# ----------------------------------------------------------------------------- bf16 helpers

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out.reshape(a.shape)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- NF4 tables

def nf4_code_table() -> np.ndarray:
    """16 NF4 values from the QLoRA quantile construction (ascending, fp32)."""
    from scipy.stats import norm

    offset = 0.9677083  # 1/2 (1 - 1/(2*15)) + 1/2 (1 - 1/(2*16)), QLoRA appendix
    positive = norm.ppf(np.linspace(offset, 0.5, 9)[:-1])
    negative = -norm.ppf(np.linspace(offset, 0.5, 8)[:-1])
    values = np.sort(np.concatenate([positive, [0.0], negative]))
    values = values / values.max()
    return values.astype(np.float32)


def dynamic_tree_map(max_exponent_bits: int = 7, total_bits: int = 8) -> np.ndarray:
    """Signed 8-bit dynamic-tree quantisation map (256 ascending fp32 values).

    For exponent level i (0..max_exponent_bits-1) the fraction interval
    [0.1, 1] is split into 2^i equal parts; the midpoints, scaled by
    10^(i - (max_exponent_bits - 1)), are taken with both signs.  0 and 1 close
    the table.
    """
    values: list[float] = []
    for i in range(max_exponent_bits):
        n = 2 ** i
        edges = np.linspace(0.1, 1.0, n + 1)
        mids = (edges[:-1] + edges[1:]) / 2.0
        scale = 10.0 ** (-(max_exponent_bits - 1) + i)
        values.extend((scale * mids).tolist())
        values.extend((-scale * mids).tolist())
    values.append(0.0)
    values.append(1.0)
    values.extend([0.0] * (2 ** total_bits - len(values)))
    return np.sort(np.asarray(values, dtype=np.float64)).astype(np.float32)


def _nearest_index_sorted(table: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Index of the nearest table value; ties resolve to the lower index."""
    t = table.astype(np.float32)
    hi = np.clip(np.searchsorted(t, x, side="left"), 1, len(t) - 1)
    lo = hi - 1
    d_lo = np.abs(x - t[lo])
    d_hi = np.abs(t[hi] - x)
    return np.where(d_hi < d_lo, hi, lo).astype(np.int64)


def nf4_thresholds(code: np.ndarray) -> np.ndarray:
    """Decision midpoints between adjacent NF4 values (fp32)."""
    c = code.astype(np.float64)
    return ((c[:-1] + c[1:]) / 2.0).astype(np.float32)


# ----------------------------------------------------------------------------- NF4 quantise / dequantise

def nf4_quantize_2d(weight: np.ndarray, blocksize: int = NF4_BLOCKSIZE,
                    nested_blocksize: int = NF4_NESTED_BLOCKSIZE,
                    code: np.ndarray | None = None, ncode: np.ndarray | None = None) -> dict:
    """Quantise one [out, in] weight the way the reference stores one expert.

    Returns the buffers of ``_store_nf4_grouped`` (experts.py:998-1031) for a
    single expert: ``packed`` uint8 [out*in/2, 1], ``absmax`` uint8 [out*in/bs],
    ``nested_absmax`` fp32 [n_nested], ``offset`` fp32 scalar, ``code`` fp32[16],
    ``nested_code`` fp32[256].
    """
    code = nf4_code_table() if code is None else code.astype(np.float32)
    ncode = dynamic_tree_map() if ncode is None else ncode.astype(np.float32)
    src = bf16_round(np.asarray(weight, dtype=np.float32)).reshape(-1)  # quant.py:327 casts to bf16
    n = src.size
    if n % blocksize:
        raise ValueError("NF4 restatement requires blocksize | numel")
    blocks = src.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = (np.float32(1.0) / absmax).astype(np.float32)
    inv = np.where(absmax == 0, np.float32(0.0), inv).astype(np.float32)
    normed = (blocks * inv[:, None]).astype(np.float32)
    mids = nf4_thresholds(code)
    q = np.searchsorted(mids, normed.reshape(-1), side="left").astype(np.uint8)  # x > mid -> upper
    packed = ((q[0::2] << 4) | q[1::2]).astype(np.uint8).reshape(-1, 1)

    # double quantisation of absmax
    offset = np.float32(np.mean(absmax.astype(np.float64)))
    centred = (absmax - offset).astype(np.float32)
    nb = nested_blocksize
    nblocks = (centred.size + nb - 1) // nb
    pad = nblocks * nb - centred.size
    cpad = np.concatenate([centred, np.zeros(pad, np.float32)]).reshape(nblocks, nb)
    nabs = np.abs(cpad).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        ninv = (np.float32(1.0) / nabs).astype(np.float32)
    ninv = np.where(nabs == 0, np.float32(0.0), ninv).astype(np.float32)
    nnormed = (cpad * ninv[:, None]).astype(np.float32).reshape(-1)[: centred.size]
    qabs = _nearest_index_sorted(ncode, nnormed).astype(np.uint8)
    return {
        "packed": packed,
        "absmax": qabs,
        "nested_absmax": nabs,
        "offset": np.asarray(offset, dtype=np.float32),
        "code": code,
        "nested_code": ncode,
        "blocksize": blocksize,
        "nested_blocksize": nested_blocksize,
    }


def nf4_absmax_dequant(absmax_q: np.ndarray, nested_absmax: np.ndarray, offset,
                       ncode: np.ndarray, nested_blocksize: int = NF4_NESTED_BLOCKSIZE) -> np.ndarray:
    """fp32 block scales: fl(fl(ncode[q] * nabsmax[b // nbs]) + offset)."""
    q = np.asarray(absmax_q, dtype=np.int64).reshape(-1)
    nabs = np.asarray(nested_absmax, dtype=np.float32).reshape(-1)
    idx = np.arange(q.size) // nested_blocksize
    prod = (ncode.astype(np.float32)[q] * nabs[idx]).astype(np.float32)
    return (prod + np.float32(offset)).astype(np.float32)


def nf4_dequantize_2d(buffers: dict, shape: tuple[int, int]) -> np.ndarray:
    """Dense bf16 values (as float32) of one expert weight."""
    code = buffers["code"].astype(np.float32)
    bs = int(buffers.get("blocksize", NF4_BLOCKSIZE))
    nbs = int(buffers.get("nested_blocksize", NF4_NESTED_BLOCKSIZE))
    scales = nf4_absmax_dequant(buffers["absmax"], buffers["nested_absmax"], buffers["offset"],
                                buffers["nested_code"], nbs)
    packed = np.asarray(buffers["packed"], dtype=np.uint8).reshape(-1)
    q = np.empty(packed.size * 2, dtype=np.int64)
    q[0::2] = packed >> 4
    q[1::2] = packed & 0xF
    vals = (code[q].reshape(-1, bs) * scales[:, None]).astype(np.float32)
    return bf16_round(vals).reshape(shape)


def nf4_quantize_grouped(weight: np.ndarray, blocksize: int = NF4_BLOCKSIZE,
                         nested_blocksize: int = NF4_NESTED_BLOCKSIZE) -> dict:
    """Per-expert NF4 quantisation of an [E, out, in] stack (experts.py:998-1031)."""
    E, out_f, in_f = weight.shape
    per = [nf4_quantize_2d(weight[e], blocksize, nested_blocksize) for e in range(E)]
    return {
        "nf4": np.stack([p["packed"] for p in per]),
        "absmax": np.stack([p["absmax"] for p in per]),
        "nabsmax": np.stack([p["nested_absmax"] for p in per]),
        "offset": np.stack([p["offset"] for p in per]).astype(np.float32),
        "code": per[0]["code"],
        "ncode": per[0]["nested_code"],
        "shape": (E, out_f, in_f),
        "blocksize": blocksize,
        "nested_blocksize": nested_blocksize,
    }


def nf4_dequantize_grouped(g: dict) -> np.ndarray:
    E, out_f, in_f = g["shape"]
    res = np.empty((E, out_f, in_f), dtype=np.float32)
    for e in range(E):
        res[e] = nf4_dequantize_2d({
            "packed": g["nf4"][e], "absmax": g["absmax"][e], "nested_absmax": g["nabsmax"][e],
            "offset": g["offset"][e], "code": g["code"], "nested_code": g["ncode"],
            "blocksize": g["blocksize"], "nested_blocksize": g["nested_blocksize"],
        }, (out_f, in_f))
    return res


# ----------------------------------------------------------------------------- INT8

def best_group_size(in_features: int, group_sizes=DEFAULT_GROUP_SIZES) -> int:
    """quant.py:87-91."""
    for g in sorted(group_sizes, reverse=True):
        if in_features % g == 0:
            return int(g)
    return 0


def hadamard(size: int) -> np.ndarray:
    """Kronecker power of the 4x4 Hadamard block, scaled by 1/sqrt(size) (quant.py:103-122)."""
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float32)
    h = h4
    cur = 4
    while cur < size:
        h = np.kron(h, h4).astype(np.float32)
        cur *= 4
    if cur != size:
        raise ValueError(f"Hadamard size must be a power of 4, got {size}")
    return (h / np.float32(math.sqrt(size))).astype(np.float32)


def rotate_last_dim(w2d: np.ndarray, group_size: int, inverse: bool) -> np.ndarray:
    """quant.py:150-178: per-group right-multiplication by H (or H^T)."""
    if group_size <= 0:
        return w2d
    out_f, in_f = w2d.shape
    h = hadamard(group_size)
    rot = h.T if inverse else h
    grouped = w2d.reshape(out_f, in_f // group_size, group_size).astype(np.float32)
    return (grouped @ rot).astype(np.float32).reshape(out_f, in_f)


def int8_quantize(weight: np.ndarray, group_size: int) -> tuple[np.ndarray, np.ndarray, int]:
    """quant.py:189-235: rotate (optional), per-row amax/127 scale, round half-even, clamp."""
    shape = weight.shape
    in_f = shape[-1]
    g = group_size if group_size > 0 and in_f % group_size == 0 else 0
    w = np.asarray(weight, dtype=np.float32).reshape(-1, in_f)
    work = rotate_last_dim(w, g, inverse=False)
    scale = np.maximum((np.abs(work).max(axis=1, keepdims=True) / np.float32(127.0)).astype(np.float32),
                       np.float32(1e-30)).astype(np.float32)
    q = np.clip(np.round((work / scale).astype(np.float32)), -127, 127).astype(np.int8)
    return q.reshape(shape), scale.reshape(*shape[:-1], 1), g


def int8_dequantize(q: np.ndarray, scale: np.ndarray, group_size: int) -> np.ndarray:
    """quant.py:238-260 (fp32 result, before the cast to the compute dtype)."""
    shape = q.shape
    in_f = shape[-1]
    work = (q.astype(np.float32) * scale.astype(np.float32)).reshape(-1, in_f).astype(np.float32)
    work = rotate_last_dim(work, group_size, inverse=True)
    return work.reshape(shape)
