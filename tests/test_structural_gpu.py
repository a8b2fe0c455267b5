"""K3/K4 parity: compaction, radix sort, Gather and regrowth on the device
against the oracle, bit for bit, plus the structural-plasticity step end to
end (small sizes against the oracle, full size through properties)."""
import numpy as np
import pytest
import torch

from plastix_b200 import _abi
from plastix_b200.runtime import (StructuralLayer, compact, gather, radix_sort_u32,
                                  regrow, sort_tail_u32)

pytestmark = pytest.mark.gpu


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def host(t, dtype=None):
    a = t.detach().cpu().numpy()
    return a.view(dtype) if dtype is not None else a


SIZES = [0, 1, 7, 4095, 4096, 4097, 100_003, 1 << 20]


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("kind", [_abi.KEEP_FLAGS, _abi.KEEP_NOT_DEAD, _abi.KEEP_ABS_GE])
def test_compact_matches_gather_of_survivors(ctx, orc, n, kind):
    rng = np.random.default_rng(n + kind)
    w = rng.normal(0, 0.1, n).astype(np.float32)
    if n > 10:
        w[3] = np.nan  # NaN is not pruned by |w| < thr
    flags = (rng.random(n) < 0.7).astype(np.uint8)
    f8 = rng.integers(0, 2**63, n, dtype=np.uint64)
    f4 = rng.integers(0, 2**32, n, dtype=np.uint32)
    f2 = rng.integers(0, 2**16, n, dtype=np.uint16)
    f1 = rng.integers(0, 256, n, dtype=np.uint8)
    if kind == _abi.KEEP_FLAGS:
        keep_src, keep = flags, flags != 0
    elif kind == _abi.KEEP_NOT_DEAD:
        keep_src, keep = flags, flags == 0
    else:
        keep_src, keep = w, orc.keep_abs_ge(w, 0.02) != 0
    srcs = [dev(x) for x in (f8, f4, f2, f1, w)]
    dsts = [torch.zeros_like(s) for s in srcs]
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    perm = torch.zeros(max(n, 1), dtype=torch.int32, device="cuda")
    compact(ctx, n, kind, dev(keep_src), list(zip(srcs, dsts)), count, threshold=0.02,
            flags=[0, 0, 0, _abi.FIELD_INC_SAT_U8, 0], perm_out=perm)
    ctx.sync()
    p = orc.survivors(keep.astype(np.uint8))
    m = int(count.item())
    assert m == p.size
    np.testing.assert_array_equal(host(perm)[:m].view(np.uint32), p.astype(np.uint32))
    for src, dst in zip((f8, f4, f2), dsts[:3]):
        np.testing.assert_array_equal(host(dst)[:m].view(src.dtype), orc.gather(p, src))
    want_age = np.minimum(orc.gather(p, f1).astype(np.int32) + 1, 255).astype(np.uint8)
    np.testing.assert_array_equal(host(dsts[3])[:m], want_age)
    np.testing.assert_array_equal(host(dsts[4])[:m].view(np.uint32),
                                  orc.gather(p, w).view(np.uint32))


@pytest.mark.parametrize("n,bits", [(0, 8), (1, 20), (4096, 12), (4097, 24),
                                    (300_001, 23), (1 << 22, 32), (50_000, 3), (10_000, 0)])
def test_radix_sort_is_stable_sort(ctx, orc, n, bits):
    rng = np.random.default_rng(n + bits)
    hi = 1 << bits if bits < 32 else 2**32
    keys = rng.integers(0, max(hi, 1), n, dtype=np.uint64).astype(np.uint32)
    if n > 100:
        keys[:50] = keys[50]  # many duplicates: stability matters
    keys_out = torch.zeros(max(n, 1), dtype=torch.int32, device="cuda")
    perm = torch.zeros(max(n, 1), dtype=torch.int32, device="cuda")
    radix_sort_u32(ctx, dev(keys) if n else torch.zeros(1, dtype=torch.int32, device="cuda")[:0],
                   keys_out, perm, 0, bits)
    ctx.sync()
    want = orc.stable_sort_perm_u32(keys)
    np.testing.assert_array_equal(host(perm)[:n].view(np.uint32), want.astype(np.uint32))
    np.testing.assert_array_equal(host(keys_out)[:n].view(np.uint32), keys[want])


def test_radix_sort_ignores_bits_outside_range(ctx, orc):
    rng = np.random.default_rng(5)
    keys = rng.integers(0, 2**32, 70_000, dtype=np.uint64).astype(np.uint32)
    keys_out = torch.zeros(keys.size, dtype=torch.int32, device="cuda")
    perm = torch.zeros(keys.size, dtype=torch.int32, device="cuda")
    radix_sort_u32(ctx, dev(keys), keys_out, perm, 4, 19)
    ctx.sync()
    want = orc.stable_sort_perm_u32((keys >> 4) & ((1 << 15) - 1))
    np.testing.assert_array_equal(host(perm).view(np.uint32), want.astype(np.uint32))


@pytest.mark.parametrize("n,n_sorted,bits,lo,hi", [
    (0, 0, 24, 0, 1), (1, 1, 24, 0, 1), (1, 0, 24, 0, 1), (5000, 5000, 24, 0, 1 << 24),
    (5000, 0, 24, 0, 1 << 24), (100_003, 84_000, 24, 0, 1 << 24),   # 16 % regrown
    (100_003, 99_999, 24, 0, 64),                                   # heavy key ties
    (300_001, 1, 23, 0, 1 << 23), (1 << 21, 1_700_000, 32, 0, 2**32),
    (77_777, 40_000, 0, 0, 1 << 20),                                # no key bits: identity
    (4096 * 3 + 5, 2048 * 5 + 1, 12, 0, 4096)])                      # partition edges
def test_sort_tail_equals_full_stable_sort(ctx, orc, n, n_sorted, bits, lo, hi):
    """plx_sort_tail_u32 (a sorted prefix, the regrown tail radix-sorted and
    merged in) gives the permutation and keys of the full stable sort, bit for
    bit, for prefixes of every length, heavy ties and partial partitions."""
    rng = np.random.default_rng(n + n_sorted + bits)
    keys = rng.integers(lo, hi, n, dtype=np.uint64).astype(np.uint32)
    mask = (1 << bits) - 1 if bits < 32 else 0xFFFFFFFF
    pre = keys[:n_sorted]
    keys[:n_sorted] = pre[np.argsort(pre & np.uint32(mask), kind="stable")]
    count = torch.tensor([n_sorted], dtype=torch.int64, device="cuda")
    keys_out = torch.zeros(max(n, 4), dtype=torch.int32, device="cuda")
    perm = torch.zeros(max(n, 4), dtype=torch.int32, device="cuda")
    k_in = dev(keys) if n else torch.zeros(4, dtype=torch.int32, device="cuda")[:0]
    sort_tail_u32(ctx, k_in, count, keys_out, perm, 0, bits)
    ctx.sync()
    want = orc.stable_sort_perm_u32(keys & np.uint32(mask))
    np.testing.assert_array_equal(host(perm)[:n].view(np.uint32), want.astype(np.uint32))
    np.testing.assert_array_equal(host(keys_out)[:n].view(np.uint32), keys[want])


def test_sort_tail_rejects_a_prefix_longer_than_the_keys(ctx):
    keys = torch.zeros(10, dtype=torch.int32, device="cuda")
    out = torch.zeros(12, dtype=torch.int32, device="cuda")
    count = torch.tensor([11], dtype=torch.int64, device="cuda")
    with pytest.raises(RuntimeError, match="exceeds"):
        sort_tail_u32(ctx, keys, count, out, out.clone(), 0, 8)


def test_gather_matches_reference_gather(ctx, orc):
    rng = np.random.default_rng(11)
    n = 123_457
    perm = rng.permutation(n).astype(np.uint32)
    fields = [rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32),
              rng.normal(size=n).astype(np.float32), rng.integers(0, 256, n, dtype=np.uint8)]
    srcs = [dev(f) for f in fields]
    dsts = [torch.empty_like(s) for s in srcs]
    gather(ctx, dev(perm), list(zip(srcs, dsts)))
    ctx.sync()
    for f, d in zip(fields, dsts):
        np.testing.assert_array_equal(host(d).view(f.dtype), orc.gather(perm, f))


def test_regrow_matches_oracle(ctx, orc):
    n, m = 50_000, 41_234
    f = np.arange(n, dtype=np.uint32)
    t = np.arange(n, dtype=np.uint32)
    w = np.ones(n, np.float32)
    age = np.full(n, 7, np.uint8)
    df, dt, dw, da = dev(f), dev(t), dev(w), dev(age)
    count = torch.tensor([m], dtype=torch.int64, device="cuda")
    regrow(ctx, count, df, dt, dw, da, src_base=3, n_src=1000, dst_base=1003, n_dst=777,
           seed=42, step_base=99)
    ctx.sync()
    wf, wt, ww, wa = orc.regrow(f, t, w, age, m, 3, 1000, 1003, 777, 42, 99)
    np.testing.assert_array_equal(host(df, np.uint32), wf)
    np.testing.assert_array_equal(host(dt, np.uint32), wt)
    np.testing.assert_array_equal(host(dw), ww)
    np.testing.assert_array_equal(host(da), wa)


def small_structural(n_src, n_dst, n, seed):
    rng = np.random.default_rng(seed)
    src = rng.integers(0, n_src, n, dtype=np.uint32)
    dst = rng.integers(0, n_dst, n, dtype=np.uint32)
    order = np.argsort(dst, kind="stable")
    f = np.ascontiguousarray(src[order])
    t = np.ascontiguousarray(dst[order] + np.uint32(n_src))
    w = rng.normal(0, 0.1, n).astype(np.float32)
    age = rng.integers(0, 256, n, dtype=np.uint8)
    act = rng.random(n_src, dtype=np.float32)
    return f, t, w, age, act


@pytest.mark.parametrize("n_src,n_dst,n", [(5000, 3000, 60_000), (1 << 16, 1 << 16, 1 << 17)])
def test_structural_steps_match_oracle(ctx, orc, n_src, n_dst, n):
    f, t, w, age, act = small_structural(n_src, n_dst, n, seed=n)
    layer = StructuralLayer(ctx, n_src, n_dst, dev(f), dev(t), dev(w), dev(age),
                            threshold=0.02, seed=7)
    act_d = dev(act)
    for step in range(3):
        out = layer.step(act_d)
        ctx.sync()
        f, t, w, age, m = orc.structural_step(f, t, w, age, n_src, n_dst, 0.02, 7, step * n)
        assert int(layer.count.item()) == m
        np.testing.assert_array_equal(host(layer.f, np.uint32), f)
        np.testing.assert_array_equal(host(layer.t, np.uint32), t)
        np.testing.assert_array_equal(host(layer.w).view(np.uint32), w.view(np.uint32))
        np.testing.assert_array_equal(host(layer.age), age)
        a_full = np.concatenate([act, np.zeros(n_dst, np.float32)])
        want, _ = orc.forward_pipeline(f, t, w, a_full, n_src)
        np.testing.assert_array_equal(host(out), want[n_src:])


def test_full_size_structural_step(ctx, orc):
    """The 16M-connection structural step (8M sources, 8M destinations):
    one step checked against the oracle bit for bit."""
    n_src = n_dst = 1 << 23
    n = 1 << 24
    g = torch.Generator(device="cuda").manual_seed(3)
    src = torch.randint(0, n_src, (n,), generator=g, device="cuda")
    dst = torch.randint(0, n_dst, (n,), generator=g, device="cuda")
    dst, order = torch.sort(dst, stable=True)
    f = src[order].to(torch.int32)
    t = (dst + n_src).to(torch.int32)
    w = torch.randn(n, generator=g, device="cuda") * 0.1
    age = torch.randint(0, 256, (n,), generator=g, device="cuda").to(torch.uint8)
    act = torch.rand(n_src, generator=g, device="cuda")
    hf, ht, hw, ha, hact = host(f, np.uint32), host(t, np.uint32), host(w), host(age), host(act)
    layer = StructuralLayer(ctx, n_src, n_dst, f, t, w, age, threshold=0.02, seed=11)
    out = layer.step(act)
    ctx.sync()
    of, ot, ow, oa, m = orc.structural_step(hf, ht, hw, ha, n_src, n_dst, 0.02, 11, 0)
    assert int(layer.count.item()) == m
    assert 0.14 * n < n - m < 0.18 * n  # ~15.9% of N(0, 0.1^2) lies within +-0.02
    tt = host(layer.t, np.uint32)
    assert np.all(np.diff(tt.astype(np.int64)) >= 0)
    np.testing.assert_array_equal(tt, ot)
    np.testing.assert_array_equal(host(layer.f, np.uint32), of)
    np.testing.assert_array_equal(host(layer.w).view(np.uint32), ow.view(np.uint32))
    np.testing.assert_array_equal(host(layer.age), oa)
    a_full = np.concatenate([hact, np.zeros(n_dst, np.float32)])
    want, _ = orc.forward_pipeline(of, ot, ow, a_full, n_src)
    np.testing.assert_array_equal(host(out), want[n_src:])


@pytest.mark.parametrize("n,dups", [(0, 0), (1, 0), (1000, 900), (500_003, 100_000),
                                    (1 << 20, 0)])
def test_proposal_sort_unique_matches_oracle(ctx, orc, n, dups):
    """DoAddConnections phases 2-3: sort CompactEdge bits, commit each once."""
    from plastix_b200.runtime import sort_unique_u64
    rng = np.random.default_rng(n + dups)
    frm = rng.integers(0, 2**32, n, dtype=np.uint64)
    to = rng.integers(0, 2**32, n, dtype=np.uint64)
    bits = (to << np.uint64(32)) | frm
    if dups and n:
        bits[rng.choice(n, dups)] = bits[rng.choice(n, dups)]
    if n >= 1000:  # the all-ones key: the reference's "previous" sentinel skips it
        bits[:3] = np.uint64(2**64 - 1)
    keys = torch.from_numpy(bits.view(np.int64)).cuda() if n else \
        torch.zeros(1, dtype=torch.int64, device="cuda")[:0]
    out = torch.zeros(max(n, 1), dtype=torch.int64, device="cuda")
    count = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    sort_unique_u64(ctx, keys, out, count)
    ctx.sync()
    want = orc.sort_unique_u64(bits)
    m = int(count.item())
    assert m == want.size
    np.testing.assert_array_equal(host(out)[:m].view(np.uint64), want)


def test_level_sort_is_stable_counting_sort(ctx, orc):
    """SortConnectionsByLevel (plastix.hpp:539-579): a stable sort of the
    connections by SrcLevel and a Gather of every field -- the radix sort on
    the 16-bit level key and plx_gather, against the oracle's stable sort."""
    rng = np.random.default_rng(12)
    n = 300_001
    level = rng.integers(0, 1024, n).astype(np.uint32)
    frm = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    w = rng.normal(size=n).astype(np.float32)
    keys_out = torch.zeros(n, dtype=torch.int32, device="cuda")
    perm = torch.zeros(n, dtype=torch.int32, device="cuda")
    radix_sort_u32(ctx, dev(level), keys_out, perm, 0, 16)
    f2, w2 = torch.empty(n, dtype=torch.int32, device="cuda"), torch.empty(n, device="cuda")
    gather(ctx, perm, [(dev(frm), f2), (dev(w), w2)])
    ctx.sync()
    want = orc.stable_sort_perm_u32(level)
    np.testing.assert_array_equal(host(perm).view(np.uint32), want.astype(np.uint32))
    np.testing.assert_array_equal(host(f2, np.uint32), orc.gather(want, frm))
    np.testing.assert_array_equal(host(w2).view(np.uint32), orc.gather(want, w).view(np.uint32))
