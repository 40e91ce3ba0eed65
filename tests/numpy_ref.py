"""Second, independent restatement (numpy, vectorised) of the reference's
activation quantisation and integer block dots, used to cross-check the C
oracle. Test infrastructure only.

float32 numpy element-wise ops round each result to binary32 (no FMA), so
these follow src/ops/quant.rs:750-771, :850-898 and :996-1057 exactly.
"""
import numpy as np


def f16(u16):
    return np.asarray(u16, np.uint16).view(np.float16).astype(np.float32)


def quantize_blocks(x):
    """x [..., 256] -> (d [...], qs int32 [..., 256])."""
    x = np.asarray(x, np.float32)
    a = np.where(x < 0, -x, x)
    a = np.where(np.isnan(a), np.float32(0), a)
    amax = a.max(axis=-1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    scaled = (x * inv[..., None]).astype(np.float32)
    bias = np.where(scaled >= 0, np.float32(0.5), np.float32(-0.5)).astype(np.float32)
    t = (scaled + bias).astype(np.float32)
    q = np.trunc(np.nan_to_num(t, nan=0.0)).clip(-127, 127).astype(np.int32)
    return d, q


def q4k_fields(w):
    """w [nb, 144] -> d, dmin, sc[nb,8], m[nb,8], q[nb,256] (element order)."""
    w = np.asarray(w, np.uint8).reshape(-1, 144)
    d = f16(w[:, 0:2].copy().view(np.uint16)[:, 0])
    dmin = f16(w[:, 2:4].copy().view(np.uint16)[:, 0])
    s = w[:, 4:16].astype(np.int32)
    sc = np.empty((len(w), 8), np.int32)
    m = np.empty((len(w), 8), np.int32)
    sc[:, :4] = s[:, 0:4] & 63
    m[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    m[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    qs = w[:, 16:].reshape(-1, 4, 32).astype(np.int32)
    q = np.concatenate([qs & 15, qs >> 4], axis=2).reshape(-1, 256)  # per half: lo32, hi32
    return d, dmin, sc, m, q


def q6k_fields(w):
    w = np.asarray(w, np.uint8).reshape(-1, 210)
    ql = w[:, 0:128].reshape(-1, 2, 64).astype(np.int32)
    qh = w[:, 128:192].reshape(-1, 2, 32).astype(np.int32)
    sc = w[:, 192:208].astype(np.int8).astype(np.int32)
    d = f16(w[:, 208:210].copy().view(np.uint16)[:, 0])
    q = np.empty((len(w), 2, 4, 32), np.int32)
    q[:, :, 0] = (ql[:, :, 0:32] & 15) | ((qh & 3) << 4)
    q[:, :, 1] = (ql[:, :, 32:64] & 15) | (((qh >> 2) & 3) << 4)
    q[:, :, 2] = (ql[:, :, 0:32] >> 4) | (((qh >> 4) & 3) << 4)
    q[:, :, 3] = (ql[:, :, 32:64] >> 4) | (((qh >> 6) & 3) << 4)
    return d, sc, q.reshape(-1, 256) - 32


def fixed_tree_rows(parts):
    """fixed_tree over the last axis, vectorised across rows."""
    p = np.asarray(parts, np.float32).copy()
    n = p.shape[-1]
    while n > 1:
        half = (n + 1) // 2
        nxt = np.empty(p.shape[:-1] + (half,), np.float32)
        pairs = n // 2
        nxt[..., :pairs] = (p[..., 0:2 * pairs:2] + p[..., 1:2 * pairs:2]).astype(np.float32)
        if n % 2:
            nxt[..., pairs] = p[..., n - 1]
        p, n = nxt, half
    return p[..., 0]


def linear_int(dtype_q6, x, w, batch, in_feat, out_feat):
    S = in_feat // 256
    x = np.asarray(x, np.float32).reshape(batch, S, 256)
    xd, xq = quantize_blocks(x)                      # [B,S], [B,S,256]
    y = np.empty((batch, out_feat), np.float32)
    if not dtype_q6:
        d, dmin, sc, m, q = q4k_fields(w)
        d, dmin = d.reshape(out_feat, S), dmin.reshape(out_feat, S)
        sc, m = sc.reshape(out_feat, S, 8), m.reshape(out_feat, S, 8)
        q = q.reshape(out_feat, S, 8, 32)
        for b in range(batch):
            xs = xq[b].reshape(S, 8, 32)
            sums = np.einsum("rsjl,sjl->rsj", q, xs)          # exact int
            bsums = xs.sum(axis=2)                            # [S,8]
            acc = (sc * sums).sum(axis=2)
            accm = (m * bsums[None]).sum(axis=2)
            t0 = ((d * xd[b][None]).astype(np.float32) * acc.astype(np.float32)).astype(np.float32)
            t1 = ((dmin * xd[b][None]).astype(np.float32) * accm.astype(np.float32)).astype(np.float32)
            y[b] = fixed_tree_rows((t0 - t1).astype(np.float32))
    else:
        d, sc, q = q6k_fields(w)
        d = d.reshape(out_feat, S)
        sc = sc.reshape(out_feat, S, 16)
        # element e -> bucket: half h = e//128, w = e%128, t = w//32, l = w%32:
        e = np.arange(256)
        bucket = 8 * (e // 128) + (e % 32) // 16 + 2 * ((e % 128) // 32)
        q = q.reshape(out_feat, S, 256)
        onehot = np.zeros((256, 16), np.int64)
        onehot[e, bucket] = 1
        for b in range(batch):
            prod = q * xq[b][None]                               # [R,S,256]
            sums = prod @ onehot                                  # [R,S,16]
            acc = (sc * sums).sum(axis=2)
            t0 = ((d * xd[b][None]).astype(np.float32) * acc.astype(np.float32)).astype(np.float32)
            y[b] = fixed_tree_rows(t0)
    return y.reshape(-1)
