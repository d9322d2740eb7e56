"""The vectorised paged-lattice writer (kv_lattice_kernel: lssab8_decode_prep_kv and lssab8_kv_append
take it for channel-contiguous, 16-byte aligned rows) against the generic per-element writer
(decode_prep_kernel, taken for every other layout -- here a channel-strided view of the same
values): int8 pages, block exponents and the sink exponent bit for bit, for bf16, fp16 and f32
inputs, dh 64 and 128, sink off and on, ragged lengths over a shuffled page table, and blocks
holding signed zeros, subnormals, infinities, NaN and values at the int8 clamp; and the in-place
rewrite of an existing lattice (build_paged_kv(out=...)) equals a fresh build."""
import pytest
import torch

from lockstep_b200 import decode as D

pytestmark = pytest.mark.gpu

LENS = [1, 17, 128, 129, 300, 700]


def _values(B, KVH, L, dh, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, KVH, L, dh, generator=g)
    x = x * torch.exp2(torch.randint(-6, 7, (B, KVH, L, 1), generator=g).float())   # rows of mixed scale
    tiny = 1e-40 if dtype != torch.float16 else 1e-6                                 # a subnormal of the dtype
    specials = torch.tensor([0.0, -0.0, tiny, -tiny, 127.5, -127.5, 126.5, float("inf"), float("-inf"),
                             float("nan")])
    # one row of block 0 and one row of the second block of every sequence get the special values;
    # key 0 (the sink's own row) gets a few as well
    for t in (5, 130):
        if t < L:
            idx = torch.randint(0, dh, (specials.numel(),), generator=g)
            x[:, :, t, idx] = specials
    x[:, :, 0, :3] = torch.tensor([-0.0, tiny, 127.5])
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dh", [128, 64])
@pytest.mark.parametrize("sink", [False, True])
def test_vectorised_writer_equals_generic_writer(dtype, dh, sink):
    B, KVH, L = len(LENS), 2, max(LENS)
    dev = torch.device("cuda")
    k = _values(B, KVH, L, dh, dtype, 1 + dh).to(dev)
    v = _values(B, KVH, L, dh, dtype, 2 + dh).to(dev)
    lens = torch.tensor(LENS, dtype=torch.int32, device=dev)
    max_pages = (L + 15) // 16 + 3
    num_pages = B * max_pages + 5
    g = torch.Generator().manual_seed(7)
    bt = torch.randperm(num_pages, generator=g)[:B * max_pages].view(B, max_pages).to(torch.int32).to(dev)
    # the same values with channel stride 2: the generic writer's layout
    k2 = torch.zeros(B, KVH, L, 2 * dh, dtype=dtype, device=dev)
    v2 = torch.zeros_like(k2)
    k2[..., ::2] = k
    v2[..., ::2] = v
    a = D.build_paged_kv(k, v, lens, bt, num_pages, sink=sink)
    b = D.build_paged_kv(k2[..., ::2], v2[..., ::2], lens, bt, num_pages, sink=sink)
    for name in ("k8p", "v8p", "ek", "ev"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    if sink:
        assert torch.equal(a.ev0, b.ev0)
    # rewriting an existing lattice in place (out=): one built from other values (K and V swapped)
    c = D.build_paged_kv(v, k, lens, bt, num_pages, sink=sink)
    c2 = D.build_paged_kv(k, v, lens, bt, num_pages, sink=sink, out=c)
    assert c2.k8p.data_ptr() == c.k8p.data_ptr()
    for name in ("k8p", "v8p", "ek", "ev") + (("ev0",) if sink else ()):
        assert torch.equal(getattr(a, name), getattr(c2, name)), name
