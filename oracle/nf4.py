"""NF4 double quantization: a quantizer to make test weights, and the dequant restatement.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Dequant (the parity target) follows solution/nf4.py:28-49 (``skc_nf4_dequant_kernel``):
for packed byte i, ``hi = b >> 4`` is the first weight and ``lo = b & 15`` the second
(solution/nf4.py:35,46-47); both fall in absmax block ``(2*i) // blocksize`` (:36);
with double quant the block scale is ``code2[absmax_u8[blk]] * absmax2[blk // blocksize2]``
then ``+ offset`` as two separately rounded fp32 operations (:38-41, launched with
``enable_fp_fusion=False`` at :443); each weight is ``code[nibble] * scale`` in fp32 (:44-45),
rounded to the output type (fp16 in the reference, :46).

Quantizer: bitsandbytes 0.50.2 (``bitsandbytes.functional.quantize_4bit``) is not installed here.
Its algorithm is restated from the published method: the NF4 data type of QLoRA
(Dettmers et al. 2023, arXiv:2305.14314, section 3 "4-bit NormalFloat") and double quantization of
the fp32 absmax values with a signed dynamic 8-bit map (Dettmers et al. 2021, arXiv:2110.02861,
"dynamic tree quantization") after subtracting their mean. The code tables are kernel INPUTS, so
dequant parity holds for any table; bit-level parity with bitsandbytes' own quantizer is unpinned.
"""

from __future__ import annotations

import numpy as np

try:  # scipy gives the normal quantile function; it is present in this image
    from scipy.stats import norm as _norm
except ImportError:  # pragma: no cover
    _norm = None


def nf4_code() -> np.ndarray:
    """The 16 NF4 values: quantiles of N(0, 1) normalised to [-1, 1], with an exact zero.

    QLoRA builds 2^(k-1) = 8 positive and 2^(k-1)-1 = 7 negative quantiles (asymmetric, so that 0
    is representable) at probabilities spread evenly between 0.5 and ``delta`` where
    delta = 1/2 (1/(2*15) + 1/(2*16)) pushed to the published offset 0.9677, then normalises by
    the largest magnitude.
    """
    if _norm is None:  # pragma: no cover
        raise RuntimeError("scipy is needed to build the NF4 table")
    offset = 0.9677083
    pos = _norm.ppf(np.linspace(offset, 0.5, 9)[:-1])      # 8 positive quantiles
    neg = -_norm.ppf(np.linspace(offset, 0.5, 8)[:-1])     # 7 negative quantiles
    values = np.sort(np.concatenate([pos, [0.0], neg]))
    values = values / np.abs(values).max()
    return values.astype(np.float32)


def dynamic_code(total_bits: int = 8, exponent_bits: int = 7) -> np.ndarray:
    """A signed dynamic (tree) 8-bit quantization map of 256 fp32 values in [-1, 1].

    Dynamic tree quantization (arXiv:2110.02861, Fig. 2): after the sign bit, a run of leading
    zero bits encodes a decimal exponent 10^-e and the bits after the first one are a linear
    fraction in (0.1, 1). Exponent level e (0 = largest magnitudes) gets 2^(bits left) fraction
    cells; each cell's value is its midpoint. Zero and +1 complete the table; it is sorted.
    """
    data: list[float] = []
    value_bits = total_bits - 1                      # one bit for the sign
    for level in range(exponent_bits):
        cells = 2 ** (level + value_bits - exponent_bits)
        edges = np.linspace(0.1, 1.0, cells + 1)
        mids = (edges[:-1] + edges[1:]) / 2.0
        mag = 10.0 ** (-(exponent_bits - 1) + level)
        data.extend((mag * mids).tolist())
        data.extend((-mag * mids).tolist())
    data.append(0.0)
    data.append(1.0)
    while len(data) < 2 ** total_bits:               # pad with zeros (never picked twice)
        data.append(0.0)
    table = np.sort(np.asarray(data[: 2 ** total_bits], dtype=np.float64))
    return table.astype(np.float32)


def _nearest(values: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Index of the nearest table entry for every value (table sorted ascending)."""
    mids = (table[1:].astype(np.float64) + table[:-1].astype(np.float64)) / 2.0
    return np.searchsorted(mids, values.astype(np.float64), side="left").astype(np.uint8)


def quantize_nf4(w: np.ndarray, blocksize: int = 64, nested: bool = True,
                 blocksize2: int = 256) -> dict:
    """Quantize a 2-D weight [N_out, K_in] (row-major) to packed NF4 with optional double quant.

    Returns a dict with the same fields as a bitsandbytes QuantState the reference reads
    (solution/nf4.py:66-85): ``packed`` uint8 [N*K/2], ``absmax`` (uint8 if nested else fp32)
    [N*K/blocksize], ``absmax2`` fp32 [ceil(n_blocks/blocksize2)], ``code`` fp32 [16],
    ``code2`` fp32 [256], ``offset`` fp32 scalar, plus ``shape``, ``blocksize``, ``blocksize2``,
    ``nested``.
    """
    w = np.asarray(w, dtype=np.float32)
    assert w.ndim == 2 and w.size % blocksize == 0 and blocksize % 2 == 0
    flat = w.reshape(-1)
    n_blocks = flat.size // blocksize
    blocks = flat.reshape(n_blocks, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax == 0, np.float32(1.0), absmax)
    code = nf4_code()
    idx = _nearest((blocks / safe[:, None]).reshape(-1), code)
    packed = ((idx[0::2] << 4) | idx[1::2]).astype(np.uint8)
    state = dict(packed=packed, code=code, shape=tuple(w.shape), blocksize=int(blocksize),
                 nested=bool(nested), blocksize2=int(blocksize2))
    if nested:
        offset = np.float32(absmax.mean(dtype=np.float64))
        centred = (absmax - offset).astype(np.float32)
        n2 = -(-n_blocks // blocksize2)
        padded = np.zeros(n2 * blocksize2, dtype=np.float32)
        padded[:n_blocks] = centred
        absmax2 = np.abs(padded.reshape(n2, blocksize2)).max(axis=1).astype(np.float32)
        absmax2 = np.where(absmax2 == 0, np.float32(1.0), absmax2).astype(np.float32)
        code2 = dynamic_code()
        scaled = centred / np.repeat(absmax2, blocksize2)[:n_blocks]
        state.update(absmax=_nearest(scaled, code2), absmax2=absmax2, code2=code2,
                     offset=np.float32(offset))
    else:
        state.update(absmax=absmax, absmax2=None, code2=None, offset=None)
    return state


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (round to nearest even) and return the 16-bit patterns."""
    bits = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequant_f32(state: dict) -> np.ndarray:
    """The fp32 products ``code[nibble] * scale`` before the final rounding, [N, K]."""
    packed = np.asarray(state["packed"], dtype=np.uint8)
    bs = int(state["blocksize"])
    n_bytes = packed.size
    byte_idx = np.arange(n_bytes, dtype=np.int64)
    block = (byte_idx * 2) // bs                                    # solution/nf4.py:36
    if state["nested"]:
        code2 = np.asarray(state["code2"], dtype=np.float32)
        absmax2 = np.asarray(state["absmax2"], dtype=np.float32)
        q = np.asarray(state["absmax"], dtype=np.uint8)[block]
        scale = code2[q] * absmax2[block // int(state["blocksize2"])]   # fp32 product, rounded
        scale = (scale + np.float32(state["offset"])).astype(np.float32)  # then the add, rounded
    else:
        scale = np.asarray(state["absmax"], dtype=np.float32)[block]
    code = np.asarray(state["code"], dtype=np.float32)
    high = code[packed >> 4] * scale                               # solution/nf4.py:44
    low = code[packed & 15] * scale                                # solution/nf4.py:45
    out = np.empty(2 * n_bytes, dtype=np.float32)
    out[0::2] = high                                               # interleave, high first (:46)
    out[1::2] = low
    return out.reshape(state["shape"])


def dequantize_nf4(state: dict, out_dtype: str = "f16") -> np.ndarray:
    """[N, K] dequantised weights; ``out_dtype`` "f16" (the reference's), "bf16" (uint16 bit
    patterns, round to nearest even) or "f32"."""
    w = dequant_f32(state)
    if out_dtype == "f16":
        return w.astype(np.float16)
    if out_dtype == "bf16":
        return f32_to_bf16_bits(w)
    if out_dtype == "f32":
        return w
    raise ValueError(out_dtype)
