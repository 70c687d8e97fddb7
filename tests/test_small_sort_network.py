"""CPU replay of k_small_sort's index arithmetic (gpu-forge_b200/csrc/
fs_kernels.cuh): the block size, pairs per thread, the pair -> element
mapping (a 0 bit inserted at log2 j), the compare direction and the claim
that a stage with j <= 32 * pp only touches the issuing warp's own elements
(so __syncwarp suffices there).  Sorting (ordered key, position) tuples with
that exact network must give the stable order for every padded size the
kernel takes."""
import numpy as np
import pytest

SMALL_BLOCK_MAX = 1024


def geometry(npad):
    block = min(max(npad // 4, 32), SMALL_BLOCK_MAX)
    pp = max(npad // (2 * block), 1)
    return block, pp, 32 * pp


def stage_pairs(npad, j):
    """(warp, i, l) of every compare-exchange of a stage, as the kernel's
    threads issue them."""
    block, pp, _ = geometry(npad)
    lj = j.bit_length() - 1
    out = []
    for tid in range(block):
        warp, lane = tid >> 5, tid & 31
        for r in range(pp):
            q = warp * 32 * pp + r * 32 + lane
            if q < npad // 2:
                i = ((q >> lj) << (lj + 1)) | (q & (j - 1))
                out.append((warp, i, i | j))
    return out


def run_network(keys, pos, npad, check_local=True):
    k = keys.copy()
    p = pos.copy()
    _, _, local_j = geometry(npad)
    kk = 2
    while kk <= npad:
        j = kk >> 1
        while j > 0:
            pairs = stage_pairs(npad, j)
            # a stage is a perfect matching of the npad elements
            touched = np.concatenate([[i for _, i, _ in pairs], [l for _, _, l in pairs]])
            assert np.array_equal(np.sort(touched), np.arange(npad))
            if check_local and j <= local_j:
                span = 2 * local_j  # elements owned by one warp
                for w, i, l in pairs:
                    assert i // span == w and l // span == w, (npad, j, w, i, l)
            for _, i, l in pairs:
                up = (i & kk) == 0
                greater = k[i] > k[l] or (k[i] == k[l] and p[i] > p[l])
                if greater == up:
                    k[i], k[l] = k[l], k[i]
                    p[i], p[l] = p[l], p[i]
            j >>= 1
        kk <<= 1
    return k, p


@pytest.mark.parametrize("npad", [2, 4, 8, 32, 64, 128, 256, 512, 1024])
def test_network_sorts_stably(npad):
    rng = np.random.default_rng(npad)
    for n in {max(npad // 2 + 1, 2), npad}:
        n = min(n, npad)
        keys = rng.integers(0, 5, n).astype(np.uint64)  # many ties
        big = np.uint64(2**64 - 1)
        k = np.concatenate([keys, np.full(npad - n, big, np.uint64)])
        p = np.concatenate([np.arange(n, dtype=np.uint64), np.full(npad - n, 2**32 - 1, np.uint64)])
        sk, sp = run_network(k, p, npad)
        order = np.argsort(keys, kind="stable")
        assert np.array_equal(sk[:n], keys[order])
        assert np.array_equal(sp[:n], order.astype(np.uint64))


@pytest.mark.parametrize("npad", [2048, 4096, 8192])
def test_large_geometry_is_warp_local(npad):
    """The sizes too slow to replay fully: the block/pair geometry and the
    warp-locality of every warp-local stage, and the block-barrier count the
    kernel comment states (15 of 78 stages at 4096)."""
    block, pp, local_j = geometry(npad)
    assert block * pp * 2 == npad and block <= SMALL_BLOCK_MAX
    span = 2 * local_j
    logn = npad.bit_length() - 1
    cross = 0
    for s in range(1, logn + 1):
        for t in range(s - 1, -1, -1):
            j = 1 << t
            if j > local_j:
                cross += 1
                continue
            pairs = stage_pairs(npad, j)
            w = np.array([x[0] for x in pairs])
            i = np.array([x[1] for x in pairs])
            l_ = np.array([x[2] for x in pairs])
            assert (i // span == w).all() and (l_ // span == w).all()
    if npad == 4096:
        assert cross == 15 and logn * (logn + 1) // 2 == 78
