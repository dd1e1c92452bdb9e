"""Steps whose items run in more than one round of CTAs, against torch fp32.

When a step has more items than the device has SMs, the persistent CTAs take
items in rounds, and the plan may pick a shallower key ring and longer chunks
(decode.cu, compute_decode_plan). Dense decode with unmerged key heads at the
config-2 shapes runs 288 items in 2 rounds with its value tiles streamed by
TMA through the ring; with two value heads per key head (Hk = 1) it streams
two gather groups per item. The reference here is the dense attention of
attention.py:64-85 in fp32 torch on the same bf16 inputs; the tolerance is the
parity tests' bf16 bar (2e-2 max-abs, 1e-2 relative RMS).

The masked case is a padded batch: with lengths down to L/2, whole chunks of
some rows are masked out, whose maximum is -inf (their weights must be 0, not
exp(-inf - -inf) = NaN). In a multi-round step each CTA's shared memory still
holds the logits of its previous item, so a chunk statistic read before all
four epilogue warps stored a tile would show up as a run-to-run difference;
every case therefore also requires two runs to be bit-identical.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, mask, scaling):
    B, Hq, _, D = q.shape
    Hk, Hv = k.shape[1], v.shape[1]
    kf = k.float().repeat_interleave(Hq // Hk, dim=1)
    vf = v.float().repeat_interleave(Hq // Hv, dim=1)
    s = torch.matmul(q.float(), kf.transpose(-1, -2)) * scaling
    if mask is not None:
        s = s + mask[..., :k.shape[2]].float()
    return torch.matmul(torch.softmax(s, dim=-1), vf)


def _close(out, ref):
    a, b = out.float(), ref
    err = (a - b).abs().max().item()
    rel = ((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt()).item()
    return err <= 2e-2 and rel <= 1e-2, (err, rel)


@pytest.mark.parametrize("Hk,Hv,masked", [(2, 2, False), (2, 2, True), (1, 2, False)])
def test_dense_multi_round_matches_fp32(Hk, Hv, masked):
    from saga_b200 import ops
    dev = torch.device("cuda", 0)
    B, L, Hq, D = 8, 32768, 12, 128
    g = torch.Generator(device=dev).manual_seed(21 + Hk + 4 * masked)
    q = (torch.randn((B, Hq, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hk, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    mask = None
    if masked:  # a padded batch: every sequence has its own length (additive mask, 0 or -inf)
        lens = torch.randint(L // 2, L + 1, (B,), generator=g, device=dev)
        keep = (torch.arange(L, device=dev)[None, :] < lens[:, None]).view(B, 1, 1, L)
        mask = torch.zeros((B, 1, 1, L), device=dev).masked_fill(~keep, float("-inf")).to(torch.bfloat16)
    scaling = D ** -0.5
    ref = _ref(q, k, v, mask, scaling)
    outs = [ops.dense_decode(q, k, v, mask, scaling) for _ in range(2)]
    torch.cuda.synchronize()
    for out in outs:
        ok, stats = _close(out, ref)
        assert ok, stats
    assert torch.equal(outs[0], outs[1])  # run-to-run identical
    assert ops.read_status(dev) & 0x1 == 0


def _pad_mask(B, L, g, dev, lo, left=False):
    lens = torch.randint(lo, L + 1, (B,), generator=g, device=dev)
    pos = torch.arange(L, device=dev)[None, :]
    keep = (pos >= (L - lens)[:, None] if left else pos < lens[:, None]).view(B, 1, 1, L)
    return torch.zeros((B, 1, 1, L), device=dev).masked_fill(~keep, float("-inf")).to(torch.bfloat16)


@pytest.mark.parametrize("op", ["dense", "calibrate", "atopn"])
def test_interleaved_steps_do_not_leak(op):
    """Step A, then step B (other queries and mask, the same caches), then A
    again, as in a decode loop: A's two results are bit-identical, so no
    state left in the CTAs' shared memory or the workspace by B reaches A."""
    from saga_b200 import ops
    dev = torch.device("cuda", 0)
    B, L, Hq, Hk, Hv, D, N = 8, 32768, 12, 2, 2, 128, 512
    g = torch.Generator(device=dev).manual_seed(77)
    k = (torch.randn((B, Hk, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    qa = (torch.randn((B, Hq, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    qb = (torch.randn((B, Hq, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    # The amortized step's stabiliser is the max of the last 256 logits
    # (attention.py:142-143): a row whose tail is masked gives NaN there as in
    # the reference, so its rows are padded on the left, as in batched
    # generation. Either way some chunks hold only a few live positions.
    left = op == "atopn"
    ma = _pad_mask(B, L, g, dev, L - 3000, left)
    mb = _pad_mask(B, L, g, dev, L // 2, left)
    thr = torch.zeros(B * Hq, device=dev, dtype=torch.float32)
    if op == "atopn":
        ops.atopn_calibrate(qa, k, v, ma, thr, N)

    def step(q, m, t):
        if op == "dense":
            return ops.dense_decode(q, k, v, m), None
        if op == "calibrate":
            return ops.atopn_calibrate(q, k, v, m, t, N), t
        return ops.atopn_decode(q, k, v, m, t, N), None

    t1, tb, t2 = thr.clone(), thr.clone(), thr.clone()
    o1, _ = step(qa, ma, t1)
    step(qb, mb, tb)
    o2, _ = step(qa, ma, t2)
    torch.cuda.synchronize()
    assert torch.isfinite(o1.float()).all()
    assert torch.equal(o1, o2)
    if op == "calibrate":
        assert torch.equal(t1, t2)
    assert ops.read_status(dev) & 0x1 == 0
