"""Layout helpers for the tests (numpy, host side)."""
import numpy as np
import torch


def hm_to_rows(n, off, ln, st, val, stride=None):
    """HM (position = row + min(d, 0)) -> rows layout [K, stride]."""
    stride = stride or (n + 31) // 32 * 32
    out = np.zeros((len(off), stride), np.float32)
    for k, d in enumerate(off):
        r0 = -min(d, 0)
        out[k, r0:r0 + ln[k]] = val[st[k]:st[k] + ln[k]]
    return out


def rows_to_hm(n, off, rows):
    ln = (n - np.abs(np.asarray(off, np.int64))).astype(np.int32)
    st = np.concatenate([[0], np.cumsum(ln[:-1], dtype=np.int64)]).astype(np.int64)
    val = np.zeros(int(ln.sum()), np.float32)
    for k, d in enumerate(off):
        r0 = -min(d, 0)
        val[st[k]:st[k] + ln[k]] = rows[k, r0:r0 + ln[k]]
    return ln, st, val


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def same(a, b):
    """Equal as floats (+0 == -0), NaN-free."""
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and bool(np.array_equal(a, b))


def rel_l2(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(a - ref) / (den if den > 0 else 1.0))
