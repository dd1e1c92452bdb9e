"""Paged caches against contiguous ones: the same logical data must give
exactly the same results (only the addresses of the rows change).

A contiguous [B, H, L, D] cache is cut into pages of page_len rows and stored
in a pool in shuffled page order; rows of a page past L, and pages no
sequence uses, hold random values, which the kernels must never use. Cases:
* the amortized step, calibration and dense decode, page_len 128 and 256,
  L not a multiple of either (bf16, tensor-core path);
* fp32 (CUDA-core scorer and P.V);
* sequences sharing their prefix pages (the prefilled prompt), each with
  its own last page, against the contiguous caches copied per sequence as
  the reference's benchmark does (speedup.py:155-160);
* the fused append of a decode token into each sequence's own last page;
* D = 64, fp16, bool and additive masks, Hk = 2 with Hv = 4, and G = 32 (the
  CUDA-core scorer);
* a page number outside the pool: SAGA_STATUS_PAGE_RANGE, no fault (the
  kernel's own check reads page 0 instead).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

B, HQ, HK, HV, D, L, N = 2, 12, 1, 2, 128, 5000, 256


def _dev():
    return torch.device("cuda", 0)


def _caches(dtype, seed=3, b=B, length=L):
    g = torch.Generator(device=_dev()).manual_seed(seed)
    q = (torch.randn((b, HQ, 1, D), generator=g, device=_dev()) * 0.5).to(dtype)
    k = (torch.randn((b, HK, length, D), generator=g, device=_dev()) * 0.5).to(dtype)
    v = (torch.randn((b, HV, length, D), generator=g, device=_dev()) * 0.5).to(dtype)
    return q, k, v


def _paginate(caches, page_len, seed=5, spare=3):
    """Pools [pages, H, page_len, D] holding every sequence's pages in a
    shuffled order, and the int32 page table [B, pages per sequence]."""
    b, _, length, _ = caches[0].shape
    npg = (length + page_len - 1) // page_len
    total = b * npg + spare
    g = torch.Generator().manual_seed(seed)
    ids = torch.randperm(total, generator=g)[: b * npg].view(b, npg)
    pools = []
    for c in caches:
        pool = torch.randn((total, c.shape[1], page_len, c.shape[3]), generator=g).to(c.dtype).to(c.device)
        for s in range(b):
            for i in range(npg):
                rows = min(page_len, length - i * page_len)
                pool[ids[s, i], :, :rows] = c[s, :, i * page_len:i * page_len + rows]
        pools.append(pool)
    return pools[0], pools[1], ids.to(torch.int32).to(caches[0].device)


def _status():
    from saga_b200 import ops
    return ops.read_status(_dev())


@pytest.mark.parametrize("page_len", [128, 256])
def test_paged_matches_contiguous_bf16(page_len):
    from saga_b200 import ops
    from saga_b200 import _lib as Lb
    q, k, v = _caches(torch.bfloat16)
    kp, vp, pt = _paginate((k, v), page_len)
    paged = dict(page_table=pt, context_len=L)
    _status()
    thr_c = torch.zeros(B * HQ, dtype=torch.float32, device=_dev())
    thr_p = torch.zeros_like(thr_c)
    out_c = ops.atopn_calibrate(q, k, v, None, thr_c, N)
    out_p = ops.atopn_calibrate(q, kp, vp, None, thr_p, N, **paged)
    assert torch.equal(thr_p, thr_c) and torch.equal(out_p, out_c)
    dc, dp = {}, {}
    out_c = ops.atopn_decode(q, k, v, None, thr_c, N, diag=dc)
    out_p = ops.atopn_decode(q, kp, vp, None, thr_c, N, diag=dp, **paged)
    torch.cuda.synchronize()
    assert torch.equal(out_p, out_c)
    assert torch.equal(dp["count"], dc["count"]) and torch.equal(dp["sel_idx"], dc["sel_idx"])
    assert torch.equal(ops.dense_decode(q, kp, vp, **paged), ops.dense_decode(q, k, v))
    assert _status() & Lb.STATUS_PAGE_RANGE == 0


def test_paged_matches_contiguous_fp32():
    from saga_b200 import ops
    q, k, v = _caches(torch.float32, length=1500)
    kp, vp, pt = _paginate((k, v), 128)
    paged = dict(page_table=pt, context_len=1500)
    thr = torch.zeros(B * HQ, dtype=torch.float32, device=_dev())
    ops.atopn_calibrate(q, k, v, None, thr, 64)
    assert torch.equal(ops.atopn_decode(q, kp, vp, None, thr, 64, **paged), ops.atopn_decode(q, k, v, None, thr, 64))
    assert torch.equal(ops.dense_decode(q, kp, vp, **paged), ops.dense_decode(q, k, v))


def test_shared_prefix_pages_and_append():
    """Four sequences decode from one prefilled prompt: its full pages are
    shared, each sequence owns a copy of the partly filled last page and
    appends its own decode token there."""
    from saga_b200 import ops
    from saga_b200 import _lib as Lb
    page_len, length, nb = 128, 1000, 4
    q1, k1, v1 = _caches(torch.bfloat16, seed=9, b=1, length=length)
    g = torch.Generator(device=_dev()).manual_seed(10)
    q = (torch.randn((nb, HQ, 1, D), generator=g, device=_dev()) * 0.5).to(torch.bfloat16)
    kn = (torch.randn((nb, HK, 1, D), generator=g, device=_dev()) * 0.5).to(torch.bfloat16)
    vn = (torch.randn((nb, HV, 1, D), generator=g, device=_dev()) * 0.5).to(torch.bfloat16)
    kp1, vp1, pt1 = _paginate((k1, v1), page_len, spare=nb)
    used = set(pt1[0].tolist())
    free = [i for i in range(kp1.shape[0]) if i not in used][:nb]
    pt = pt1.repeat(nb, 1)
    for s in range(nb):  # own copy of the last (partly filled) page
        kp1[free[s]] = kp1[pt1[0, -1]]
        vp1[free[s]] = vp1[pt1[0, -1]]
        pt[s, -1] = free[s]
    # contiguous reference: the prompt copied per sequence
    k = k1.repeat(nb, 1, 1, 1).contiguous()
    v = v1.repeat(nb, 1, 1, 1).contiguous()
    _status()
    thr = torch.zeros(nb * HQ, dtype=torch.float32, device=_dev())
    thr_p = torch.zeros_like(thr)
    out_c = ops.atopn_calibrate(q, k, v, None, thr, N, k_new=kn, v_new=vn, append_pos=length - 1)
    out_p = ops.atopn_calibrate(q, kp1, vp1, None, thr_p, N, k_new=kn, v_new=vn, append_pos=length - 1,
                                page_table=pt, context_len=length)
    assert torch.equal(out_p, out_c) and torch.equal(thr_p, thr)
    row = (length - 1) % page_len
    for s in range(nb):
        assert torch.equal(kp1[pt[s, -1], :, row], kn[s, :, 0]) and torch.equal(vp1[pt[s, -1], :, row], vn[s, :, 0])
    assert torch.equal(kp1[pt1[0, 0]], k1[0, :, :page_len])  # the shared pages are untouched
    out_c = ops.atopn_decode(q, k, v, None, thr, N)
    out_p = ops.atopn_decode(q, kp1, vp1, None, thr, N, page_table=pt, context_len=length)
    torch.cuda.synchronize()
    assert torch.equal(out_p, out_c)
    assert _status() & Lb.STATUS_PAGE_RANGE == 0


def test_page_number_outside_pool_sets_status():
    from saga_b200 import ops
    from saga_b200 import _lib as Lb
    q, k, v = _caches(torch.bfloat16, length=600)
    kp, vp, pt = _paginate((k, v), 128)
    pt[1, 2] = kp.shape[0] + 7  # past the pool: the kernel reads page 0 instead and reports it
    _status()
    ops.dense_decode(q, kp, vp, page_table=pt, context_len=600)
    assert _status() & Lb.STATUS_PAGE_RANGE


@pytest.mark.parametrize("dtype,d,hq,hk,hv,mask_kind", [
    (torch.bfloat16, 64, 8, 2, 4, "bool"),       # D = 64, two key heads, more value heads
    (torch.float16, 128, 12, 1, 2, "additive"),  # fp16 with an additive mask
    (torch.bfloat16, 128, 32, 1, 2, None),       # G = 32: CUDA-core scorer
])
def test_paged_configurations(dtype, d, hq, hk, hv, mask_kind):
    """Other kernel configurations through the page table, against the
    contiguous run (bit-exact), with masks read at logical positions."""
    from saga_b200 import ops
    b, length, n = 2, 1700, 64
    g = torch.Generator(device=_dev()).manual_seed(21)
    q = (torch.randn((b, hq, 1, d), generator=g, device=_dev()) * 0.5).to(dtype)
    k = (torch.randn((b, hk, length, d), generator=g, device=_dev()) * 0.5).to(dtype)
    v = (torch.randn((b, hv, length, d), generator=g, device=_dev()) * 0.5).to(dtype)
    mask = None
    if mask_kind == "bool":
        mask = torch.rand((b, 1, 1, length), generator=g, device=_dev()) > 0.1
    elif mask_kind == "additive":
        mask = torch.where(torch.rand((b, hq, 1, length), generator=g, device=_dev()) > 0.1, 0.0, -1e4).to(dtype)
    kp, vp, pt = _paginate((k, v), 256)
    paged = dict(page_table=pt, context_len=length)
    thr = torch.zeros(b * hq, dtype=torch.float32, device=_dev())
    thr_p = torch.zeros_like(thr)
    assert torch.equal(ops.atopn_calibrate(q, kp, vp, mask, thr_p, n, **paged), ops.atopn_calibrate(q, k, v, mask, thr, n))
    assert torch.equal(thr_p, thr)
    assert torch.equal(ops.atopn_decode(q, kp, vp, mask, thr, n, **paged), ops.atopn_decode(q, k, v, mask, thr, n))
    assert torch.equal(ops.dense_decode(q, kp, vp, mask, **paged), ops.dense_decode(q, k, v, mask))
