"""Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers:
as easy as 1, 2, 3", SC'11) in numpy: the test-side restatement of the
generator the attention kernels use for dropout keep decisions."""
import numpy as np

M0, M1 = 0xD2511F53, 0xCD9E8D57
W0, W1 = 0x9E3779B9, 0xBB67AE85
U32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised over numpy arrays of uint32 counters; key (k0, k1) ints."""
    c = [np.asarray(x, dtype=np.uint64) & U32 for x in (c0, c1, c2, c3)]
    k0, k1 = np.uint64(k0 & 0xFFFFFFFF), np.uint64(k1 & 0xFFFFFFFF)
    for _ in range(10):
        p0 = c[0] * np.uint64(M0)
        p1 = c[2] * np.uint64(M1)
        hi0, lo0 = p0 >> np.uint64(32), p0 & U32
        hi1, lo1 = p1 >> np.uint64(32), p1 & U32
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = (k0 + np.uint64(W0)) & U32
        k1 = (k1 + np.uint64(W1)) & U32
    return [x.astype(np.uint32) for x in c]


def dropout_keep(elems, p, seed, offset=0):
    """Keep decisions of elements e (row * Kn + slot), as the kernels take them."""
    e = np.asarray(elems, dtype=np.uint64)
    r = philox4x32_10(e >> np.uint64(2), e >> np.uint64(34), np.full_like(e, offset & 0xFFFFFFFF),
                      np.full_like(e, (offset >> 32) & 0xFFFFFFFF), seed & 0xFFFFFFFF, seed >> 32)
    w = np.choose((e & np.uint64(3)).astype(np.int64), r)
    t = min(int(p * 4294967296.0), 0xFFFFFFFF)
    return w >= np.uint32(t)
