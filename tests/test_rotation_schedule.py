"""The chain-sharing schedule of the reference-order rotation kernel (ref_rotate16_kernel in
csrc/rotate_quant.cu), restated in numpy fp32 on the host: sixteen outputs jl + 16*i of one
thread carried as (block sign) * acc, classes of outputs sharing one chain while their block
multipliers agree (rep16), must give every output exactly the bits of its own sequential chain
acc = fl(acc + sign(j, k) * x_k), k = 0..255 (the reference's OpenBLAS order for rows of 5+
groups), with 2,736 fused adds per sixteen outputs."""

import numpy as np

F32 = np.float32


def h4(a, b):
    return -1.0 if a + b == 3 else 1.0


def sign(j, k):
    s = 1.0
    for d in range(4):
        s *= h4((j >> 2 * d) & 3, (k >> 2 * d) & 3)
    return s


def sequential_chain(x, j):
    acc = F32(0)
    for k in range(256):
        acc = F32(acc + F32(sign(j, k)) * x[k])
    return acc


def rep16(i, b):
    a, c = i & 3, i >> 2
    if b == 0:
        return 0
    if b == 1:
        return 0 if a < 2 else 2
    if b < 4:
        return a
    if b < 8:
        return a + 4 * (0 if c < 2 else 2)
    return i


def sig16(i, b):
    return h4(i & 3, b & 3) * h4(i >> 2, b >> 2)


def shared_chains(x, jl):
    lam = [h4(jl >> 2, l >> 2) * h4(jl & 3, l & 3) for l in range(16)]
    acc = [F32(0)] * 16
    adds = 0
    for b in range(16):
        if b > 0:
            old = list(acc)
            for i in range(16):
                if rep16(i, b) == i:
                    acc[i] = F32(old[rep16(i, b - 1)] * F32(sig16(i, b) * sig16(i, b - 1)))
        for i in range(16):
            if rep16(i, b) != i:
                continue
            for l in range(16):
                acc[i] = F32(acc[i] + x[16 * b + l] * F32(lam[l]))  # = fma(x, +-1, acc)
                adds += 1
    return [F32(acc[i] * F32(sig16(i, 15))) for i in range(16)], adds


def test_classes_share_exactly_what_the_sequential_chains_share():
    rng = np.random.default_rng(0)
    cases = [(rng.standard_normal(256) * 10.0 ** rng.uniform(-3, 3)).astype(F32),
             np.where(np.arange(256) % 3 == 0, F32(-1e-3), F32(1e-3)).astype(F32)]  # many ties of magnitude
    for x in cases:
        for jl in (0, 5, 10, 15):
            got, adds = shared_chains(x, jl)
            assert adds == 2736
            for i in range(16):
                want = sequential_chain(x, jl + 16 * i)
                assert got[i] == want and (got[i] != 0 or want == 0), (jl, i)
                if got[i] != 0:
                    assert got[i].view(np.uint32) == want.view(np.uint32), (jl, i)


def test_class_members_have_equal_multipliers_at_every_block_change():
    """The invariant behind rep16: within a class, every member's carried multiplier at the
    change into block b equals the representative's, and classes only split (never merge)."""
    for b in range(1, 16):
        for i in range(16):
            r = rep16(i, b)
            assert sig16(i, b) * sig16(i, b - 1) == sig16(r, b) * sig16(r, b - 1), (i, b)
            assert rep16(r, b - 1) == rep16(i, b - 1), (i, b)
