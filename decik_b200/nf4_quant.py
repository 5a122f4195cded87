"""NF4 double quantization on the host, to make NF4 weights for random-init models and benches.

bitsandbytes (``quantize_4bit``) is not a dependency; this restates the published method:
NF4 (QLoRA, arXiv:2305.14314): 16 quantiles of N(0, 1) normalised to [-1, 1] with an exact 0,
per-block absmax scaling (blocksize 64), weights mapped to the nearest code and packed two per
byte, first weight in the high nibble; double quant: the fp32 absmax values minus their mean,
per-256-block absmax, mapped to a signed dynamic 8-bit map (arXiv:2110.02861). The result has the
fields of a bitsandbytes QuantState (packed, absmax, code, absmax2, code2, offset, blocksize,
blocksize2, nested, shape).
"""

from __future__ import annotations

import numpy as np


def _ppf(p: np.ndarray) -> np.ndarray:
    from scipy.stats import norm
    return norm.ppf(p)


def nf4_code() -> np.ndarray:
    offset = 0.9677083
    pos = _ppf(np.linspace(offset, 0.5, 9)[:-1])
    neg = -_ppf(np.linspace(offset, 0.5, 8)[:-1])
    values = np.sort(np.concatenate([pos, [0.0], neg]))
    return (values / np.abs(values).max()).astype(np.float32)


def dynamic_code(total_bits: int = 8, exponent_bits: int = 7) -> np.ndarray:
    data = []
    value_bits = total_bits - 1
    for level in range(exponent_bits):
        cells = 2 ** (level + value_bits - exponent_bits)
        edges = np.linspace(0.1, 1.0, cells + 1)
        mids = (edges[:-1] + edges[1:]) / 2.0
        mag = 10.0 ** (-(exponent_bits - 1) + level)
        data.extend((mag * mids).tolist())
        data.extend((-mag * mids).tolist())
    data += [0.0, 1.0]
    data += [0.0] * (2 ** total_bits - len(data))
    return np.sort(np.asarray(data[: 2 ** total_bits])).astype(np.float32)


def _nearest(values, table):
    mids = (table[1:].astype(np.float64) + table[:-1].astype(np.float64)) / 2.0
    return np.searchsorted(mids, values.astype(np.float64), side="left").astype(np.uint8)


def quantize_nf4(w, blocksize: int = 64, nested: bool = True, blocksize2: int = 256) -> dict:
    w = np.asarray(w, dtype=np.float32)
    flat = w.reshape(-1)
    n_blocks = flat.size // blocksize
    blocks = flat.reshape(n_blocks, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax == 0, np.float32(1.0), absmax)
    code = nf4_code()
    idx = _nearest((blocks / safe[:, None]).reshape(-1), code)
    st = dict(packed=((idx[0::2] << 4) | idx[1::2]).astype(np.uint8), code=code, shape=tuple(w.shape),
              blocksize=int(blocksize), nested=bool(nested), blocksize2=int(blocksize2))
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
        st.update(absmax=_nearest(scaled, code2), absmax2=absmax2, code2=code2, offset=offset)
    else:
        st.update(absmax=absmax, absmax2=None, code2=None, offset=None)
    return st
