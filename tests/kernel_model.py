"""Numpy model of the tensor-core decode kernel's fixed-point arithmetic.

The sm_100a decode kernel (K2) runs both contractions of a packed page on the
INT8 tensor cores (``tcgen05.mma.kind::i8``):

* QK: integer Key codes (u8, 0..255; INT2/INT4 codes masked in place, so
  they carry a power-of-two weight w_c that the B row divides out) times the
  per-page products ``q_j[c] * scale_c / w_c`` written as fixed point ``X``
  (|X| <= 2^29) relative to a power-of-two block exponent (one per query group
  and page), offset by 2^30 so the four limbs (bytes) are unsigned.  The
  token's code sum n_t (the byte sum of its code words, computed on the CUDA
  cores) removes the offset exactly:
  ``acc0 + 2^8 acc1 + 2^16 acc2 + 2^24 (acc3 - 64 n_t)``.
* PV: integer Value codes (u8, 0..3) times ``p_t * vscale_t`` written as 23-bit
  unsigned fixed point (three limbs) relative to a per-page exponent (the page's
  largest Value scale: p <= 1 after the max update).

This model reproduces that arithmetic (integer parts exactly, float parts in
fp32) so the scheme's error against the oracle can be measured on the CPU;
``test_kernel_model.py`` pins it inside the decode tolerance.
"""
from __future__ import annotations

import numpy as np

from oracle import packed_ref as orc


def _exp2_ceil(x: np.ndarray) -> np.ndarray:
    """Smallest power-of-two exponent e with |x| <= 2^e (x > 0)."""
    m, e = np.frexp(np.asarray(x, np.float64))
    return np.where(m == 0.5, e - 1, e).astype(np.int64)


def model_attention(layer: orc.OracleLayer, query: np.ndarray, key_new, value_new, scaling: float,
                    qk_bits: int = 29, pv_bits: int = 23) -> np.ndarray:
    """Decode attention of ``query`` ``[n_q, D]`` over ``layer`` (page size 128,
    k_group 128, v_group D) computed with the kernel's fixed-point scheme for
    the packed history and fp32 for the residual.  Returns ``[n_q, D]``."""
    tab = layer.table
    H, D = tab["tier"].shape
    n_q = query.shape[0]
    gq = n_q // H
    T = layer.hist_len
    out = np.zeros((n_q, D))
    kh, vh = layer.dequantize() if T else (None, None)
    for h in range(H):
        q = query[h * gq:(h + 1) * gq].astype(np.float32)        # [gq, D]
        # one block exponent for the whole query group: max_j,c |q_j[c]| <= 2^eq
        eq = np.full(gq, int(_exp2_ceil(max(float(np.abs(q).max()), 1e-30))))
        m = np.full(gq, -np.inf)
        l = np.zeros(gq)
        o = np.zeros((gq, D))
        for pg in range(T // 128):
            t0 = pg * 128
            s_int = np.zeros((128, gq))
            bias = np.zeros(gq)
            scale_max = 0.0
            tiers = []
            for code, bits in orc.TIER_BITS:
                cnt = int(tab[code]["count"][h])
                if cnt == 0:
                    continue
                idx = tab[code]["index"][h, :cnt]
                codes = orc.unpack_ints(layer.hist_k[code]["code"][h, t0:t0 + 128], cnt, bits)
                sc = layer.hist_k[code]["scale"][h, :cnt, pg].astype(np.float32)
                mn = layer.hist_k[code]["min"][h, :cnt, pg].astype(np.float32)
                # codes masked in place: INT2 slot 4i+k carries 4^k, INT4 slot 2i+k carries 16^k
                slots = np.arange(cnt)
                weight = 4 ** (slots % 4) if bits == 2 else 16 ** (slots % 2) if bits == 4 else np.ones(cnt, np.int64)
                tiers.append((idx, codes, sc, mn, weight))
                scale_max = max(scale_max, float(sc.max()))
            esc = int(_exp2_ceil(scale_max))
            for idx, codes, sc, mn, weight in tiers:
                # X = rint(q * 2^(qk_bits - eq) / w * (scale * 2^-esc)), |X| <= 2^qk_bits
                qq = (q[:, idx] * np.ldexp(np.float32(1), (qk_bits - eq))[:, None]).astype(np.float32)
                qq = (qq / weight.astype(np.float32)[None, :]).astype(np.float32)
                sp = (sc * np.float32(2.0 ** -esc)).astype(np.float32)
                X = np.rint((qq * sp[None, :]).astype(np.float32)).astype(np.int64)   # [gq, cnt]
                U = X + (1 << (qk_bits + 1))
                assert U.min() >= 0 and U.max() < (1 << 31)
                A = codes.astype(np.int64) * weight[None, :]
                assert A.max() <= 255
                acc = [A @ ((U >> (8 * k)) & 0xFF).T for k in range(4)]
                n_t = A.sum(axis=1)[:, None]
                s_int += (acc[0] + 256.0 * acc[1] + 65536.0 * acc[2] + 16777216.0 * acc[3]
                          - float(1 << (qk_bits + 1)) * n_t)
                bias += (q[:, idx].astype(np.float64) @ mn.astype(np.float64))
            scale_qk = np.ldexp(1.0, eq + esc - qk_bits)            # per q-head
            s = s_int * scale_qk[None, :] + bias[None, :]
            cnt16 = int(tab[3]["count"][h])
            if cnt16:
                idx16 = tab[3]["index"][h, :cnt16]
                k16 = layer.hist_k[3]["value"][h, t0:t0 + 128, :cnt16].astype(np.float32)
                s += k16.astype(np.float64) @ q[:, idx16].T.astype(np.float64)
            s = s * scaling                                           # [128, gq]
            pm = s.max(axis=0)
            m_new = np.maximum(m, pm)
            alpha = np.where(np.isinf(m), 0.0, np.exp(m - m_new))
            p = np.exp(s - m_new[None, :])
            vs = layer.hist_v["scale"][h, t0:t0 + 128, 0].astype(np.float64)
            vm = layer.hist_v["min"][h, t0:t0 + 128, 0].astype(np.float64)
            vcodes = orc.unpack_ints(layer.hist_v["code"][h, t0:t0 + 128], D, 2).astype(np.int64)
            # p <= 1 after the max update, so p * vscale <= max vscale: one exponent per page.
            ev = np.full(gq, int(_exp2_ceil(np.maximum(vs.max(), 1e-30))))
            U = np.minimum(np.rint(p * vs[:, None] * np.ldexp(1.0, pv_bits - ev)[None, :]),
                           (1 << pv_bits) - 1).astype(np.int64)
            acc = sum(((U >> (8 * k)) & 0xFF).T @ vcodes * 256.0 ** k for k in range((pv_bits + 7) // 8))
            o = o * alpha[:, None] + acc * np.ldexp(1.0, ev - pv_bits)[:, None] + (p * vm[:, None]).sum(0)[:, None]
            l = l * alpha + p.sum(axis=0)
            m = m_new
        # residual + new token in fp64
        rk = [np.zeros((0, D))] if layer.tail_k is None else [layer.tail_k[h]]
        rv = [np.zeros((0, D))] if layer.tail_v is None else [layer.tail_v[h]]
        rk.append(np.asarray(key_new, np.float64)[h])
        rv.append(np.asarray(value_new, np.float64)[h])
        rk, rv = np.concatenate(rk), np.concatenate(rv)
        s = (rk @ q.T.astype(np.float64)) * scaling
        pm = s.max(axis=0)
        m_new = np.maximum(m, pm)
        alpha = np.where(np.isinf(m), 0.0, np.exp(m - m_new))
        p = np.exp(s - m_new[None, :])
        o = o * alpha[:, None] + p.T @ rv
        l = l * alpha + p.sum(axis=0)
        out[h * gq:(h + 1) * gq] = o / l[:, None]
    del kh, vh
    return out
