"""Each CUDA kernel alone against its plain PyTorch twin, at sizes other than the engine's."""

import math
from types import SimpleNamespace

import pytest
import torch

from torch_kernels import TorchKernels

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16]


@pytest.fixture(scope="module")
def kernels():
    from tt_transformers_b200.kernels import load_kernels

    return load_kernels("cuda:0")


@pytest.fixture(scope="module")
def twin():
    return TorchKernels("cuda:0")


def tol(dtype):
    return 2e-5 if dtype == torch.float32 else 2e-2


def close(got, ref, dtype, scale=None):
    ref = ref.float()
    err = float((got.float() - ref).abs().max())
    bound = tol(dtype) * (scale if scale is not None else max(1.0, float(ref.abs().max())))
    assert err <= bound, f"max error {err} > {bound}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("vocab,width,tokens", [(300, 80, 17), (1000, 2048, 5), (77, 9, 3)])
def test_embedding(kernels, twin, dtype, vocab, width, tokens):
    g = torch.Generator(device="cuda").manual_seed(0)
    table = torch.randn(vocab, width, device="cuda", generator=g).to(dtype)
    ids = torch.randint(0, vocab, (tokens,), device="cuda", generator=g, dtype=torch.int32)
    assert torch.equal(kernels.embedding(table, ids), twin.embedding(table, ids))


@pytest.mark.parametrize("dtype", DTYPES)
def test_embedding_with_a_scale_and_softcap(kernels, twin, dtype):
    g = torch.Generator(device="cuda").manual_seed(2)
    for vocab, width in ((50, 24), (301, 100), (64, 1027)):           # widths with and without the 16-byte path
        table = torch.randn(vocab, width, device="cuda", generator=g).to(dtype)
        ids = torch.randint(0, vocab, (13,), device="cuda", generator=g, dtype=torch.int32)
        got = kernels.embedding(table, ids, 5.5)
        assert torch.allclose(got, table[ids.long()].float() * 5.5, rtol=1e-6, atol=0)
    for rows, cols, cap in ((3, 1000, 30.0), (1, 128256, 50.0), (70, 33, 2.5)):
        logits = torch.randn(rows, cols + 5, device="cuda", generator=g) * 3 * cap
        view = logits[:, :cols]                                       # rows further apart than their length
        want = cap * torch.tanh(view.double() / cap)
        untouched = logits[:, cols:].clone()
        kernels.softcap(view, cap)
        assert float((view.double() - want).abs().max()) <= 2e-6 * cap
        assert torch.equal(logits[:, cols:], untouched)
        assert float(view.abs().max()) <= cap


def test_embedding_flags_bad_token(kernels):
    from tt_transformers_b200.kernels import EngineDeviceError

    table = torch.randn(10, 8, device="cuda")
    out = kernels.embedding(table, torch.tensor([3, 12], device="cuda", dtype=torch.int32))
    assert torch.equal(out[1], torch.zeros(8, device="cuda"))
    with pytest.raises(EngineDeviceError):
        kernels.check_status()
    kernels.check_status()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,width,eps,wdtype", [(5, 96, 1e-6, None), (33, 2048, 1e-5, torch.float32),
                                                     (2, 7, 1e-3, None), (3, 8192, 1e-5, None)])
def test_add_rmsnorm(kernels, twin, dtype, rows, width, eps, wdtype):
    g = torch.Generator(device="cuda").manual_seed(1)
    res = torch.randn(rows, width, device="cuda", generator=g) * 3
    delta = torch.randn(rows, width, device="cuda", generator=g).to(dtype)
    weight = (1 + 0.1 * torch.randn(width, device="cuda", generator=g)).to(wdtype or dtype)
    for d in (delta, None):
        r1, r2 = res.clone(), res.clone()
        got = kernels.add_rmsnorm(r1, d, weight, eps, dtype)
        ref = twin.add_rmsnorm(r2, d, weight, eps, torch.float32)
        close(r1, r2, torch.float32)
        close(got, ref, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,inter", [(3, 320), (17, 200), (1, 8192), (64, 13)])
def test_swiglu(kernels, twin, dtype, rows, inter):
    g = torch.Generator(device="cuda").manual_seed(2)
    x = (torch.randn(rows, 2 * inter, device="cuda", generator=g) * 3).to(dtype)
    close(kernels.swiglu(x), twin.swiglu(x.float()), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("width", [96, 2048, 7])
def test_gather_rows(kernels, dtype, width):
    x = torch.randn(20, width, device="cuda").to(dtype)
    rows = torch.tensor([19, 0, 7, 7, 3], device="cuda", dtype=torch.int32)
    assert torch.equal(kernels.gather_rows(x, rows), x[rows.long()])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M,N,K", [(1, 384, 96), (3, 100, 320), (8, 3072, 2048), (5, 77, 41), (9, 96, 64),
                                   (50, 320, 96), (130, 200, 80), (64, 257, 1000), (200, 2048, 512),
                                   (2, 2048, 8192), (16, 1000, 72), (17, 33, 8), (32, 2048, 2048), (64, 3072, 2048),
                                   (7, 128256, 256), (40, 50, 1000)])
def test_linear(kernels, dtype, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(dtype)
    ref = x.double() @ w.double().t()
    close(kernels.linear(x, w), ref, dtype)
    got32 = kernels.linear(x, w, out_dtype=torch.float32)
    assert got32.dtype == torch.float32
    close(got32, ref, torch.float32 if dtype == torch.float32 else torch.bfloat16,
          scale=None if dtype == torch.float32 else 0.05)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M,inter,K", [(1, 320, 96), (8, 8192, 2048), (5, 200, 80), (20, 136, 72), (33, 1000, 256),
                                       (64, 512, 128), (70, 320, 96), (3, 77, 41)])
def test_linear_swiglu(kernels, twin, dtype, M, inter, K):
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) / math.sqrt(K) * 2).to(dtype)
    ref = twin.linear_swiglu(x.double(), w.double())
    close(kernels.linear_swiglu(x, w), ref, dtype)


def make_paged_case(dtype, heads, kv_heads, head_dim, page_size, segments, window=None, seed=0, num_pages=None):
    """Random qkv for the new tokens of several segments and a cache that already holds
    each segment's earlier keys and values on shuffled pages."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(n for _, n in segments)
    num_pages = num_pages or sum(-(-(p + n) // page_size) for p, n in segments) + 3
    qkv = torch.randn(T, (heads + 2 * kv_heads) * head_dim, device="cuda", generator=g).to(dtype)
    keys = torch.randn(num_pages + 1, kv_heads, page_size, head_dim, device="cuda", generator=g).to(dtype)
    values = torch.randn(num_pages + 1, kv_heads, page_size, head_dim, device="cuda", generator=g).to(dtype)
    perm = (torch.randperm(num_pages, generator=torch.Generator().manual_seed(seed)) + 1).tolist()
    W = max(-(-(p + n) // page_size) for p, n in segments)
    table = torch.zeros(len(segments), W, dtype=torch.int32)
    for r, (p, n) in enumerate(segments):
        for i in range(-(-(p + n) // page_size)):
            table[r, i] = perm.pop()
    positions = torch.tensor([p + i for p, n in segments for i in range(n)], dtype=torch.int32, device="cuda")
    seg_of = torch.tensor([r for r, (p, n) in enumerate(segments) for _ in range(n)], dtype=torch.int32, device="cuda")
    cu = [0]
    for _, n in segments:
        cu.append(cu[-1] + n)
    batch = SimpleNamespace(positions=positions, seg_of_token=seg_of, seg_lens=[n for _, n in segments],
                            seg_pos0_list=[p for p, _ in segments], num_segments=len(segments),
                            cu_seqlens=torch.tensor(cu, dtype=torch.int32, device="cuda"),
                            seg_pos0=torch.tensor([p for p, _ in segments], dtype=torch.int32, device="cuda"),
                            max_seg_len=max(n for _, n in segments), max_context=max(p + n for p, n in segments),
                            extras={})
    view = SimpleNamespace(keys=keys, values=values, block_table=table.cuda(), page_size=page_size, window=window)
    return qkv, batch, view


ATTN_CASES = [
    # heads, kv_heads, head_dim, page_size, segments (cached before, new tokens), window
    (4, 2, 16, 4, [(0, 7), (13, 1), (5, 3)], None),
    (3, 1, 32, 8, [(0, 33), (40, 1)], None),
    (5, 5, 48, 16, [(0, 2), (130, 1), (17, 20), (255, 1)], None),
    (8, 2, 64, 16, [(300, 1), (0, 140)], None),
    (2, 1, 128, 16, [(100, 5)], None),
    (4, 2, 16, 4, [(0, 40), (37, 1), (20, 9)], 11),
    (6, 3, 80, 8, [(9, 30)], 16),
    # head sizes of the tensor-core kernel: 64-row tiles, 16-row tiles, key splits, windows, odd group sizes
    (8, 2, 64, 16, [(0, 200), (70, 33), (500, 1)], None),
    (8, 2, 64, 16, [(900, 1), (17, 1), (0, 1), (333, 1)], None),
    (4, 1, 64, 8, [(1000, 3)], None),
    (3, 1, 128, 16, [(0, 100), (129, 40)], None),
    (6, 2, 128, 16, [(700, 1), (63, 1), (64, 1)], None),
    (8, 8, 64, 4, [(0, 130), (300, 2)], None),
    (8, 2, 64, 16, [(0, 150), (400, 1), (90, 20)], 100),
    (32, 8, 64, 16, [(2000, 1)], None),
    (10, 2, 64, 16, [(50, 70)], None),
    # the tcgen05 kernel at head size 128 and with heads per KV head that do not divide 128
    (32, 8, 128, 16, [(0, 300), (1000, 37)], None),
    (24, 8, 128, 16, [(0, 130), (700, 50), (64, 64)], None),
    (12, 4, 64, 32, [(0, 257), (3000, 43)], None),
    (7, 1, 128, 8, [(0, 90), (500, 30)], None),
    (8, 2, 64, 128, [(0, 300), (200, 100)], None),                 # pages larger than a key tile
    (8, 4, 128, 256, [(0, 70), (250, 20), (256, 30)], None),
]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", ATTN_CASES)
def test_rope_kv_write_and_attention(kernels, twin, dtype, case):
    heads, kv_heads, head_dim, page_size, segments, window = case
    qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, page_size, segments, window)
    inv_freq = (1.0 / (10000.0 ** (torch.arange(0, head_dim, 2).float() / head_dim))).cuda()
    qkv2 = qkv.clone()
    view2 = SimpleNamespace(keys=view.keys.clone(), values=view.values.clone(), block_table=view.block_table,
                            page_size=page_size, window=window)
    kernels.rope_kv_write(qkv, batch, inv_freq, head_dim, heads, kv_heads, head_dim, view, True)
    twin.rope_kv_write(qkv2, batch, inv_freq, head_dim, heads, kv_heads, head_dim, view2, True)
    q_cols = heads * head_dim
    close(qkv[:, :q_cols], qkv2[:, :q_cols], dtype)
    close(view.keys, view2.keys, dtype)
    assert torch.equal(view.values, view2.values)
    scale = head_dim ** -0.5
    got = kernels.paged_attention(qkv, batch, heads, kv_heads, head_dim, scale, view)
    ref = twin.paged_attention(qkv2.float(), batch, heads, kv_heads, head_dim, scale,
                               SimpleNamespace(keys=view2.keys.float(), values=view2.values.float(),
                                               block_table=view.block_table, page_size=page_size, window=window))
    close(got, ref, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_partial_rotation_and_no_rotation(kernels, twin, dtype):
    heads, kv_heads, head_dim, page_size = 4, 2, 32, 8
    for rotary_dim in (16, 0):
        qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, page_size, [(3, 9), (20, 1)], seed=5)
        inv_freq = (1.0 / (10000.0 ** (torch.arange(0, max(rotary_dim, 2), 2).float() / max(rotary_dim, 2)))).cuda()
        qkv2 = qkv.clone()
        view2 = SimpleNamespace(keys=view.keys.clone(), values=view.values.clone(), block_table=view.block_table,
                                page_size=page_size, window=None)
        kernels.rope_kv_write(qkv, batch, inv_freq if rotary_dim else None, rotary_dim, heads, kv_heads, head_dim, view)
        twin.rope_kv_write(qkv2, batch, inv_freq, rotary_dim, heads, kv_heads, head_dim, view2)
        close(qkv[:, :heads * head_dim], qkv2[:, :heads * head_dim], dtype)
        close(view.keys, view2.keys, dtype)
        assert torch.equal(view.values, view2.values)


@pytest.mark.parametrize("dtype", DTYPES)
def test_rotation_of_neighbouring_pairs(kernels, twin, dtype):
    """`interleaved`: pair (2i, 2i + 1) instead of (i, i + d/2). Against the twin, and against what the reference's
    own pair-swap matrix gives on rows in its interleaved order (tests/golden/make_golden.py)."""
    import os

    for heads, kv_heads, head_dim, rotary_dim in ((4, 2, 32, 32), (3, 1, 64, 64), (2, 2, 48, 16)):
        qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, 8, [(3, 9), (20, 1)], seed=6)
        inv_freq = (1.0 / (10000.0 ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim))).cuda()
        qkv2 = qkv.clone()
        view2 = SimpleNamespace(keys=view.keys.clone(), values=view.values.clone(), block_table=view.block_table,
                                page_size=8, window=None)
        kernels.rope_kv_write(qkv, batch, inv_freq, rotary_dim, heads, kv_heads, head_dim, view, interleaved=True)
        twin.rope_kv_write(qkv2, batch, inv_freq, rotary_dim, heads, kv_heads, head_dim, view2, interleaved=True)
        close(qkv[:, :heads * head_dim], qkv2[:, :heads * head_dim], dtype)
        close(view.keys, view2.keys, dtype)
        assert torch.equal(view.values, view2.values)
    if dtype != torch.float32:
        return
    golden = torch.load(os.path.join(os.path.dirname(__file__), "golden", "reference_parts.pt"))
    heads, hd = golden["rope_heads"], golden["rope_head_dim"]
    q = (golden["rope_x"] @ golden["rope_w"].T).view(3, heads, hd)           # the checkpoint's row order
    meta = torch.stack([q[..., :hd // 2], q[..., hd // 2:]], dim=-1).flatten(-2)   # the reference's interleaved order
    qkv = torch.cat([meta.reshape(3, heads * hd), torch.zeros(3, 2 * hd)], 1).cuda().contiguous()
    batch = SimpleNamespace(positions=golden["rope_pos"].to(torch.int32).cuda(),
                            seg_of_token=torch.zeros(3, dtype=torch.int32, device="cuda"))
    kernels.rope_kv_write(qkv, batch, golden["rope_inv_freq"].cuda(), hd, heads, 1, hd, None, write_kv=False,
                          interleaved=True)
    assert torch.allclose(qkv[:, :heads * hd].cpu().view(3, heads, hd), golden["rope_rotated_meta"], atol=1e-5)


def test_attention_finds_a_far_key(kernels):
    """One key among hundreds is made to stand out; the output must be its value."""
    heads, kv_heads, head_dim, page_size = 2, 1, 64, 16
    for dtype in DTYPES:
        for far in (0, 15, 16, 127, 128, 129, 383, 500):
            qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, page_size, [(511, 1)], seed=far)
            q = torch.zeros(head_dim, device="cuda")
            q[3] = 40.0
            qkv.view(1, heads + 2, head_dim)[0, :heads] = q.to(dtype)
            page = int(view.block_table[0, far // page_size])
            view.keys[:, :, :, 3] = 0
            view.keys[page, 0, far % page_size, 3] = 40.0
            got = kernels.paged_attention(qkv, batch, heads, kv_heads, head_dim, 1.0, view)
            want = view.values[page, 0, far % page_size].float()
            for h in range(heads):
                close(got.view(heads, head_dim)[h], want, dtype)


DECODE_CASES = [
    # heads, kv_heads, head_dim, page_size, segments (cached before, new tokens), window
    (32, 8, 64, 16, [(8191, 1), (0, 1), (63, 1), (64, 1), (65, 1), (4095, 1)], None),
    (8, 8, 64, 8, [(100, 1), (7, 1), (8, 2), (511, 5), (1024, 8)], None),          # one head per group, up to 8 tokens
    (6, 2, 64, 32, [(1000, 1), (31, 2), (32, 1)], None),                           # three heads per group
    (10, 2, 64, 64, [(700, 1), (63, 3)], None),                                    # five per group: 16-row tiles
    (16, 1, 64, 128, [(1500, 1), (127, 1), (128, 1)], None),                       # sixteen per group, pages beyond a tile
    (8, 2, 128, 16, [(3000, 1), (15, 1), (16, 1), (200, 2)], None),
    (24, 2, 128, 8, [(900, 1), (64, 1)], None),                                    # twelve per group at head size 128
    (8, 2, 64, 16, [(500, 1), (99, 1), (100, 1), (101, 2), (10, 1)], 100),         # windows
    (4, 1, 128, 32, [(2000, 1), (300, 3)], 257),
    (8, 4, 64, 256, [(1000, 1), (255, 1), (256, 1)], 300),
    (4, 2, 64, 16, [(20000, 1), (16383, 1), (16384, 2)], None),                    # more pages than a block keeps in shared memory
]


@pytest.mark.parametrize("case", DECODE_CASES)
@pytest.mark.parametrize("tma", [True, False])
def test_decode_attention(kernels, twin, case, tma):
    """Both decode kernels (TMA loads with transposed products; the mma.sync kernel's decode shape) against
    the plain reference, with one split and with several. Every cache slot that no query may see (slots
    past a segment's end, keys a window has passed, pages of nobody) holds NaN: none may reach the output."""
    heads, kv_heads, head_dim, page_size, segments, window = case
    dtype = torch.bfloat16
    qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, page_size, segments, window, seed=3)
    visible = torch.zeros(view.keys.shape[0], page_size, dtype=torch.bool)
    for r, (p, n) in enumerate(segments):
        low = max(0, p - window + 1) if window else 0
        for key in range(low, p + n):
            visible[int(view.block_table[r, key // page_size]), key % page_size] = True
    ref = twin.paged_attention(qkv.float(), batch, heads, kv_heads, head_dim, 0.3,
                               SimpleNamespace(keys=view.keys.float(), values=view.values.float(),
                                               block_table=view.block_table, page_size=page_size, window=window))
    hidden = (~visible).cuda()[:, None, :, None].expand_as(view.keys)
    view.keys[hidden] = float("nan")
    view.values[hidden] = float("nan")
    before = kernels.use_tma_decode
    kernels.use_tma_decode = tma
    try:
        for splits in (None, 1, 3, 16, 20, 40):     # 16: the largest cluster; 20, 40: partial results and the merge kernel
            batch.extras.clear()
            if splits is not None:
                plan = kernels._attention_plan(batch, heads // kv_heads, kv_heads, head_dim)
                assert plan[0], "the case is meant for the decode kernels"
                key = ("attention_plan", heads // kv_heads, kv_heads, head_dim, False)
                batch.extras[key] = plan[:4] + (splits,)
            got = kernels.paged_attention(qkv, batch, heads, kv_heads, head_dim, 0.3, view)
            assert not torch.isnan(got.float()).any()
            close(got, ref, dtype)
        kernels.check_status()
    finally:
        kernels.use_tma_decode = before


@pytest.mark.parametrize("case", [
    (8, 2, 64, 16, [(0, 200), (70, 33), (500, 40)], None),          # the TMA + tcgen05 kernel's geometry
    (32, 8, 64, 16, [(0, 300), (1000, 37)], None),
    (8, 2, 64, 16, [(0, 150), (90, 20)], 100),                      # a window: the mma.sync kernel
    (3, 1, 128, 16, [(0, 100), (129, 40)], None),
    (32, 8, 128, 16, [(0, 200), (1100, 45)], None),
    (6, 3, 80, 8, [(9, 30)], 16),                                   # the kernel for any size
])
def test_prompt_attention_ignores_slots_that_hold_nothing(kernels, twin, case):
    """Prompt portions: cache slots past a segment's end or below its window, and pages of nobody, hold NaN."""
    heads, kv_heads, head_dim, page_size, segments, window = case
    dtype = torch.bfloat16
    qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, page_size, segments, window, seed=8)
    visible = torch.zeros(view.keys.shape[0], page_size, dtype=torch.bool)
    for r, (p, n) in enumerate(segments):
        low = max(0, p - window + 1) if window else 0
        for key in range(low, p + n):
            visible[int(view.block_table[r, key // page_size]), key % page_size] = True
    ref = twin.paged_attention(qkv.float(), batch, heads, kv_heads, head_dim, 0.3,
                               SimpleNamespace(keys=view.keys.float(), values=view.values.float(),
                                               block_table=view.block_table, page_size=page_size, window=window))
    hidden = (~visible).cuda()[:, None, :, None].expand_as(view.keys)
    view.keys[hidden] = float("nan")
    view.values[hidden] = float("nan")
    got = kernels.paged_attention(qkv, batch, heads, kv_heads, head_dim, 0.3, view)
    assert not torch.isnan(got.float()).any()
    close(got, ref, dtype)
    kernels.check_status()


@pytest.mark.parametrize("case", [
    (8, 2, 64, 16, [(0, 200), (70, 33), (500, 40)]),
    (32, 8, 64, 16, [(0, 700), (3000, 300), (17, 1), (255, 2)]),      # long blocks, a block of one row group
    (8, 8, 64, 8, [(0, 513), (100, 257)]),                             # one head per KV head: 256 tokens a block
    (6, 2, 64, 32, [(0, 90), (1000, 170)]),                            # three heads per KV head: 85 tokens a block
    (24, 8, 128, 16, [(0, 130), (700, 50), (64, 64)]),
    (32, 8, 128, 16, [(0, 300), (2100, 140)]),
    (16, 1, 128, 64, [(0, 40), (500, 33)]),                            # sixteen heads per KV head, pages of 64
    (8, 2, 64, 256, [(0, 300), (200, 100)]),                           # pages larger than a key tile
])
def test_prompt_attention_with_key_splits(kernels, twin, case):
    """The tcgen05 attention kernel against plain attention, with the number of key splits the host would choose
    and with 2, 3 and 5 (partial results and the merge kernel); long blocks, blocks of a single row group, heads
    per KV head that do not divide a tile; every cache slot that no query may see holds NaN."""
    heads, kv_heads, head_dim, page_size, segments = case
    dtype = torch.bfloat16
    qkv, batch, view = make_paged_case(dtype, heads, kv_heads, head_dim, page_size, segments, None, seed=12)
    visible = torch.zeros(view.keys.shape[0], page_size, dtype=torch.bool)
    for r, (p, n) in enumerate(segments):
        for key in range(p + n):
            visible[int(view.block_table[r, key // page_size]), key % page_size] = True
    ref = twin.paged_attention(qkv.float(), batch, heads, kv_heads, head_dim, 0.25,
                               SimpleNamespace(keys=view.keys.float(), values=view.values.float(),
                                               block_table=view.block_table, page_size=page_size, window=None))
    hidden = (~visible).cuda()[:, None, :, None].expand_as(view.keys)
    view.keys[hidden] = float("nan")
    view.values[hidden] = float("nan")
    for splits in (None, 2, 3, 5):
        batch.extras.clear()
        if splits is not None:
            plan = kernels._attention_plan(batch, heads // kv_heads, kv_heads, head_dim, big_tiles=True)
            batch.extras[("attention_plan", heads // kv_heads, kv_heads, head_dim, True)] = plan[:4] + (splits,)
        got = kernels.paged_attention(qkv, batch, heads, kv_heads, head_dim, 0.25, view)
        assert not torch.isnan(got.float()).any(), splits
        close(got, ref, dtype)
        kernels.check_status()


@pytest.mark.parametrize("vocab,rows", [(384, 5), (128256, 3), (1000, 64), (33, 2)])
def test_sample(kernels, twin, vocab, rows):
    g = torch.Generator(device="cuda").manual_seed(4)
    logits = torch.randn(rows, vocab, device="cuda", generator=g) * 3
    logits[0, 7] = logits[0, 20] = logits[0].max() + 1      # equal maxima: the lower id wins
    assert torch.equal(kernels.sample(logits).cpu(), twin.sample(logits).cpu())
    assert int(kernels.sample(logits)[0]) == 7
    temperature = torch.full((rows,), 0.8, device="cuda")
    temperature[-1] = 0.0
    seeds = torch.arange(rows, device="cuda", dtype=torch.int64) * 7919 + 1
    for counter in range(4):
        counters = torch.full((rows,), counter, device="cuda", dtype=torch.int32)
        for top_k, top_p in ((0, 1.0), (5, 1.0), (40, 0.7), (1, 1.0), (64, 0.2), (0, 0.9), (100, 1.0), (90, 0.6), (0, 0.3)):
            if top_k > vocab:
                continue
            k = torch.full((rows,), top_k, device="cuda", dtype=torch.int32)
            p = torch.full((rows,), top_p, device="cuda")
            got = kernels.sample(logits, temperature, k, p, seeds, counters).cpu()
            ref = twin.sample(logits, temperature, k, p, seeds, counters).cpu()
            agree = (got == ref).float().mean()
            # a draw that lands within rounding of a bin edge may fall either way
            assert agree >= 0.9, (top_k, top_p, got.tolist(), ref.tolist())
    for s, c in ((0, 0), (1, 5), (2 ** 40 + 3, 77)):
        assert abs(kernels.uniform(s, c) - twin.uniform(s, c)) < 1e-7


def test_sample_draws_exactly_from_the_sets_the_references_host_sampler_allows(kernels):
    """2,000 draws per setting on fixed logits: every drawn token is one the reference's _select may draw
    (src/tt_transformers/models/hf_generation.py:138-146; the sets were taken from that function), every allowed
    token of some weight is drawn, and the frequencies follow its probabilities. Settings: top_p over the whole
    vocabulary, top_k beyond the kernel's candidate list, both together, and the candidate-list path."""
    import os

    golden = torch.load(os.path.join(os.path.dirname(__file__), "golden", "reference_parts.pt"))
    logits, draws = golden["allowed_logits"], 2000
    settings = {(c["top_k"], c["top_p"]) for c in golden["allowed"]}
    assert {(0, 0.9), (100, 1.0), (50, 0.8)} <= settings
    for case in golden["allowed"]:
        for row in range(logits.shape[0]):
            rows = logits[row][None].repeat(draws, 1).cuda()
            picks = kernels.sample(rows, torch.full((draws,), case["temperature"], device="cuda"),
                                   torch.full((draws,), case["top_k"], dtype=torch.int32, device="cuda"),
                                   torch.full((draws,), case["top_p"], device="cuda"),
                                   torch.full((draws,), 4242 + row, dtype=torch.int64, device="cuda"),
                                   torch.arange(draws, dtype=torch.int32, device="cuda")).cpu().long()
            freq = torch.bincount(picks, minlength=logits.shape[1]).float() / draws
            allowed, probs = case["mask"][row], case["probs"][row]
            what = (case["temperature"], case["top_k"], case["top_p"], row)
            assert not bool(((freq > 0) & ~allowed).any()), what              # nothing outside the set
            assert bool((freq > 0)[probs >= 0.006].all()), what               # (1 - 0.006)^2000 = 6e-6
            assert float((freq - probs).abs().sum()) / 2 < 0.08, what         # total variation


@pytest.mark.parametrize("vocab", [33, 257, 5000, 128256])
def test_sample_top_k_with_many_equal_logits(kernels, twin, vocab):
    """top_k up to the candidate list's length is found slice by slice (a radix select per slice, then per row).
    Logits rounded to halves give long runs of equal values at every cut: the k largest with the lowest ids first
    among equals, exactly as the plain twin picks them."""
    g = torch.Generator(device="cuda").manual_seed(vocab)
    rows = 4 if vocab > 10000 else 40
    logits = torch.round(torch.randn(rows, vocab, device="cuda", generator=g) * 2) / 2
    logits[1] = 0.0                                           # every logit equal: the first k ids
    logits[2, ::3] = float("-inf")
    temperature = torch.full((rows,), 1.3, device="cuda")
    seeds = torch.arange(rows, device="cuda", dtype=torch.int64) * 31 + 7
    for top_k, top_p in ((1, 1.0), (2, 1.0), (7, 1.0), (33, 0.8), (50, 1.0), (64, 0.5)):
        for counter in range(3):
            counters = torch.full((rows,), counter, device="cuda", dtype=torch.int32)
            k = torch.full((rows,), top_k, device="cuda", dtype=torch.int32)
            p = torch.full((rows,), top_p, device="cuda")
            got = kernels.sample(logits, temperature, k, p, seeds, counters).cpu()
            ref = twin.sample(logits, temperature, k, p, seeds, counters).cpu()
            # a draw within rounding of a bin's edge may fall either way; the sets must be the same, so most picks are
            assert float((got == ref).float().mean()) >= 0.9, (top_k, top_p, got.tolist(), ref.tolist())
            assert int(got[1]) < min(top_k, vocab)            # all equal: one of the first k ids
    # rows of one batch with every kind of setting: greedy, the whole vocabulary, a short list, a long one, top_p alone
    kinds = [(0.0, 0, 1.0), (0.9, 0, 1.0), (0.9, 5, 1.0), (0.9, min(100, vocab), 1.0), (0.9, 0, 0.7), (0.9, 64, 0.9)]
    t = torch.tensor([x[0] for x in kinds], device="cuda")
    k = torch.tensor([x[1] for x in kinds], device="cuda", dtype=torch.int32)
    p = torch.tensor([x[2] for x in kinds], device="cuda")
    mixed = torch.randn(len(kinds), vocab, device="cuda", generator=g) * 2
    sd = torch.arange(len(kinds), device="cuda", dtype=torch.int64) + 100
    same = 0
    for counter in range(5):
        c = torch.full((len(kinds),), counter, device="cuda", dtype=torch.int32)
        got, ref = kernels.sample(mixed, t, k, p, sd, c).cpu(), twin.sample(mixed, t, k, p, sd, c).cpu()
        assert int(got[0]) == int(ref[0])
        same += int((got == ref).sum())
    assert same >= 27


def test_sample_distribution(kernels):
    """Draws over many counters follow softmax(logits / temperature)."""
    logits = torch.tensor([[0.0, 1.0, 2.0, 3.0, -50.0]], device="cuda").repeat(4096, 1)
    temperature = torch.full((4096,), 1.5, device="cuda")
    seeds = torch.full((4096,), 1234, device="cuda", dtype=torch.int64)
    counters = torch.arange(4096, device="cuda", dtype=torch.int32)
    got = kernels.sample(logits, temperature, None, None, seeds, counters)
    freq = torch.bincount(got.long().cpu(), minlength=5).float() / 4096
    expect = torch.softmax(logits[0].cpu() / 1.5, 0)
    assert float((freq - expect).abs().max()) < 0.03


@pytest.mark.parametrize("dtype,head_dim", [(torch.float32, 32), (torch.bfloat16, 32), (torch.bfloat16, 64)])
def test_attention_does_not_follow_a_page_id_outside_the_pool(kernels, dtype, head_dim):
    """A block-table entry that points outside the pool is flagged and its keys are left out;
    nothing outside the pool is read."""
    from tt_transformers_b200.kernels import EngineDeviceError

    qkv, batch, view = make_paged_case(dtype, 4, 2, head_dim, 16, [(100, 1), (40, 3)], seed=11)
    kernels.check_status()
    view.block_table[0, 2] = view.keys.shape[0] + 5
    view.block_table[1, 0] = -3
    out = kernels.paged_attention(qkv, batch, 4, 2, head_dim, 0.2, view)
    assert not torch.isnan(out.float()).any()
    with pytest.raises(EngineDeviceError, match="page id"):
        kernels.check_status()
    kernels.check_status()


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (65, 128, 64), (130, 200, 72), (256, 384, 96), (300, 320, 1000),
                                   (2048, 3072, 2048), (512, 2048, 8192), (100, 1000, 8)])
def test_tcgen05_product(kernels, M, N, K):
    """The TMA + tcgen05 matrix product against a float64 product, with tails in every dimension."""
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    ref = x.double() @ w.double().t()
    before = kernels.use_tcgen05
    kernels.use_tcgen05 = True
    try:
        got = kernels.linear(x, w)
        got32 = kernels.linear(x, w, out_dtype=torch.float32)
        kernels.check_status()            # raises if a wait inside the kernel gave up
    finally:
        kernels.use_tcgen05 = before
    close(got, ref, torch.bfloat16)
    assert got32.dtype == torch.float32
    close(got32, ref, torch.bfloat16)


@pytest.mark.parametrize("M,inter,K", [(128, 128, 64), (200, 320, 96), (70, 136, 72), (1024, 1024, 512)])
def test_tcgen05_product_with_swiglu(kernels, twin, M, inter, K):
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) / math.sqrt(K) * 2).to(torch.bfloat16)
    ref = twin.linear_swiglu(x.double(), w.double())
    before = kernels.use_tcgen05
    kernels.use_tcgen05 = True
    try:
        got = kernels.linear_swiglu(x, w)
        kernels.check_status()
    finally:
        kernels.use_tcgen05 = before
    close(got, ref, torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(17, 320, 96), (24, 2048, 8192), (33, 257, 1000), (64, 3072, 2048), (64, 2048, 8192),
                                   (1, 130, 72), (50, 6, 264), (64, 128256, 256), (40, 200, 4104), (64, 128, 2112)])
def test_tcgen05_product_that_streams_the_weights(kernels, twin, M, N, K):
    """gemm_skinny_tcgen05.cu (17 to 64 rows; it takes fewer too): widths that are no multiple of its tiles, a
    reduction that is no multiple of its k-block, every cluster size from 1 to 8 (few row tiles and a long K
    give the most slices; with K = 2,112 the last of eight slices is empty), both output types, and the SwiGLU form."""
    g = torch.Generator(device="cuda").manual_seed(10)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K) * 2).to(torch.bfloat16)
    before = (kernels.SKINNY_TCGEN05_MIN_ROWS, kernels.SKINNY_TCGEN05_MIN_K, kernels.use_skinny_tcgen05)
    kernels.SKINNY_TCGEN05_MIN_ROWS = kernels.SKINNY_TCGEN05_MIN_K = 0      # every product of up to 64 rows goes there
    kernels.use_skinny_tcgen05 = True
    try:
        launches = kernels.launches
        got = kernels.linear(x, w)
        got32 = kernels.linear(x, w, out_dtype=torch.float32)
        fused = kernels.linear_swiglu(x, w) if N % 2 == 0 else None
        assert kernels.launches - launches == (3 if N % 2 == 0 else 2), "one launch of this package's kernels per product"
        kernels.check_status()            # raises if a wait inside the kernel gave up
    finally:
        kernels.SKINNY_TCGEN05_MIN_ROWS, kernels.SKINNY_TCGEN05_MIN_K, kernels.use_skinny_tcgen05 = before
    ref = x.double() @ w.double().t()
    close(got, ref, torch.bfloat16)
    assert got32.dtype == torch.float32
    close(got32, ref, torch.bfloat16)
    if fused is not None:
        close(fused, twin.linear_swiglu(x.double(), w.double()), torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(1, 2048, 2048), (8, 8192, 2048), (5, 1000, 1544), (7, 520, 264), (2, 100, 48),
                                   (8, 2048, 8192), (3, 6, 4104), (8, 3072, 3072), (4, 160, 24576)])
def test_persistent_product_that_streams_the_weights_through_a_ring(kernels, twin, M, N, K):
    """gemv_ring.cu (up to 8 rows): every kind of product it may be given (plain with either output type, the
    SwiGLU pair) whether the engine routes that kind there or not; widths with fewer rows than blocks and with rows
    no multiple of a tile, a reduction that is no multiple of a step of 512, x in shared memory (short K) and from
    global memory (long K). The other skinny kernel is the second opinion beside float64."""
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K) * 2).to(torch.bfloat16)
    before = kernels.ring_gemv, kernels.RING_SWIGLU_MIN_ROWS
    try:
        kernels.ring_gemv, kernels.RING_SWIGLU_MIN_ROWS = 15, 1
        launches = kernels.launches
        got = kernels.linear(x, w)
        got32 = kernels.linear(x, w, out_dtype=torch.float32)
        fused = kernels.linear_swiglu(x, w) if N % 2 == 0 else None
        assert kernels.launches - launches == (3 if N % 2 == 0 else 2), "one launch of this package's kernels per product"
        kernels.ring_gemv = 0
        other = kernels.linear(x, w)
    finally:
        kernels.ring_gemv, kernels.RING_SWIGLU_MIN_ROWS = before
    ref = x.double() @ w.double().t()
    close(got, ref, torch.bfloat16)
    assert got32.dtype == torch.float32
    close(got32, ref, torch.bfloat16)
    close(got, other, torch.bfloat16)
    if fused is not None:
        close(fused, twin.linear_swiglu(x.double(), w.double()), torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(17, 320, 96), (32, 2048, 2048), (40, 100, 1000), (64, 3072, 2048), (64, 2048, 8192)])
def test_skinny_tensor_core_product_at_all_its_row_counts(kernels, twin, M, N, K):
    """The mma.sync weight-streaming kernel takes up to 64 rows, although the engine hands it 16 at most."""
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    before = kernels.TENSOR_SKINNY_ROWS, kernels.SKINNY_ROWS, kernels.use_skinny_tcgen05
    kernels.TENSOR_SKINNY_ROWS, kernels.SKINNY_ROWS, kernels.use_skinny_tcgen05 = 64, 64, False
    try:
        launches = kernels.launches
        got = kernels.linear(x, w)
        assert kernels.launches == launches + 1, "the product ran on this package's kernel"
        if N % 2 == 0:
            fused = kernels.linear_swiglu(x, w)
    finally:
        kernels.TENSOR_SKINNY_ROWS, kernels.SKINNY_ROWS, kernels.use_skinny_tcgen05 = before
    close(got, x.double() @ w.double().t(), torch.bfloat16)
    if N % 2 == 0:
        close(fused, twin.linear_swiglu(x.double(), w.double()), torch.bfloat16)


@pytest.mark.parametrize("heads,kv_heads,head_dim,page_size,segments,width", [
    (8, 2, 64, 16, [(300, 1), (0, 1), (17, 1)], 128), (32, 8, 64, 16, [(8000, 1)] * 8, 2048),
    (6, 2, 128, 8, [(63, 1), (64, 1)], 96), (4, 4, 16, 4, [(5, 1), (6, 1), (7, 1), (0, 1), (100, 1)], 72),
    (3, 1, 32, 8, [(40, 1)], 96), (8, 2, 64, 16, [(10 * i + 3, 1) for i in range(13)], 264),
    (6, 2, 128, 8, [(7 * i, 1) for i in range(16)], 512),
    (8, 2, 64, 16, [(11 * i + 1, 1) for i in range(23)], 2048), (6, 2, 128, 8, [(5 * i, 1) for i in range(64)], 520),
    (5, 1, 32, 8, [(3 * i + 2, 1) for i in range(40)], 96), (32, 8, 64, 16, [(100 + i, 1) for i in range(33)], 2048)])
def test_fused_qkv_projection_rotation_and_cache_write(kernels, twin, heads, kv_heads, head_dim, page_size, segments, width):
    """One kernel for a decode step's QKV product, rotation and cache write against the three steps one by one."""
    _, batch, view = make_paged_case(torch.bfloat16, heads, kv_heads, head_dim, page_size, segments, seed=21)
    g = torch.Generator(device="cuda").manual_seed(22)
    M = len(segments)
    x = torch.randn(M, width, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((heads + 2 * kv_heads) * head_dim, width, device="cuda", generator=g) / math.sqrt(width)).to(torch.bfloat16)
    inv_freq = (1.0 / (500000.0 ** (torch.arange(0, head_dim, 2).float() / head_dim))).cuda()
    view2 = SimpleNamespace(keys=view.keys.float(), values=view.values.float(), block_table=view.block_table,
                            page_size=page_size, window=None)
    q = kernels.fused_qkv_rope(x, w, batch, inv_freq, head_dim, heads, kv_heads, head_dim, view, True)
    assert q is not None and q.shape == (M, heads * head_dim)
    qkv = (x.float() @ w.float().t())                     # float32 product, then the twin's rotation and write
    twin.rope_kv_write(qkv, batch, inv_freq, head_dim, heads, kv_heads, head_dim, view2, True)
    close(q, qkv[:, :heads * head_dim], torch.bfloat16)
    close(view.keys, view2.keys, torch.bfloat16)
    close(view.values, view2.values, torch.bfloat16)
    kernels.check_status()


@pytest.fixture
def fusing(kernels):
    """The kernel table with the norm and residual fusions of the skinny products switched on."""
    before = kernels.fuse_norm, kernels.fuse_add
    kernels.fuse_norm = kernels.fuse_add = True
    yield kernels
    kernels.fuse_norm, kernels.fuse_add = before


class _Norm:
    """As much of a norm part as the fused products ask for."""

    def __init__(self, weight, eps):
        self.weight, self.eps = weight, eps

    def fusion_args(self):
        return self.weight.float().contiguous(), self.eps


def _rms(residual, weight, eps):
    r = residual.double()
    return r * torch.rsqrt((r * r).mean(-1, keepdim=True) + eps) * weight.double()


@pytest.mark.parametrize("M,N,K,eps", [(1, 384, 96, 1e-5), (8, 2048, 2048, 1e-5), (5, 72, 80, 1e-6), (16, 2048, 2048, 1e-5),
                                       (12, 256, 8192, 1e-3), (8, 8192, 2048, 1e-5), (3, 104, 4096, 1e-5)])
def test_skinny_products_take_the_residual_add_and_the_norm_between_them(fusing, twin, M, N, K, eps):
    """The product that ends a sub-layer adds to the float32 stream and prepares the norm that follows;
    the product after it (plain, SwiGLU pair, both output types) finishes that norm. Against the steps
    one by one in float64."""
    from tt_transformers_b200.parts.base import ADDED, DeferredNorm

    kernels = fusing
    g = torch.Generator(device="cuda").manual_seed(31)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    stream = torch.randn(M, N, device="cuda", generator=g) * 3.0
    weight = 1.0 + 0.3 * torch.randn(N, device="cuda", generator=g)
    norm = _Norm(weight.to(torch.bfloat16), eps)
    want_stream = stream.double() + x.double() @ w.double().t()
    # the add alone
    alone = stream.clone()
    assert kernels.linear(x, w, accumulate=alone) is ADDED
    close(alone, want_stream, torch.bfloat16)
    # the add with the norm prepared
    prepared = kernels.linear(x, w, accumulate=stream, next_norm=norm)
    assert isinstance(prepared, DeferredNorm) and prepared.made_for is norm
    close(stream, want_stream, torch.bfloat16)
    normed = _rms(stream, norm.weight, eps)            # of the stream as the kernel left it
    close(prepared.materialize(), normed, torch.bfloat16)
    w2 = (torch.randn(320, N, device="cuda", generator=g) / math.sqrt(N)).to(torch.bfloat16)
    for out_dtype in (torch.bfloat16, torch.float32):
        got = kernels.linear(prepared, w2, out_dtype=out_dtype)
        assert got.dtype == out_dtype
        close(got, normed @ w2.double().t(), torch.bfloat16)
    close(kernels.linear_swiglu(prepared, w2), twin.linear_swiglu(normed, w2.double()), torch.bfloat16)
    # finished by a product that also ends a sub-layer
    stream2 = torch.randn(M, 320, device="cuda", generator=g)
    want2 = stream2.double() + normed @ w2.double().t()
    assert kernels.linear(prepared, w2, accumulate=stream2) is ADDED
    close(stream2, want2, torch.bfloat16)


def test_products_that_cannot_fuse_fall_back_to_the_steps_one_by_one(fusing):
    """More rows than the skinny kernel takes, or float32: the product comes back for the caller to add,
    and a DeferredNorm that reaches such a product is materialised."""
    from tt_transformers_b200.parts.base import DeferredNorm

    kernels = fusing
    g = torch.Generator(device="cuda").manual_seed(32)
    for dtype, M in ((torch.bfloat16, 40), (torch.float32, 4)):
        x = torch.randn(M, 96, device="cuda", generator=g).to(dtype)
        w = (torch.randn(64, 96, device="cuda", generator=g) / 10).to(dtype)
        stream = torch.zeros(M, 64, device="cuda")
        out = kernels.linear(x, w, accumulate=stream, next_norm=_Norm(torch.ones(64, device="cuda", dtype=dtype), 1e-5))
        assert torch.is_tensor(out) and float(stream.abs().max()) == 0.0
        calls = []

        def materialize():
            calls.append(1)
            return x

        got = kernels.linear(DeferredNorm(x, torch.zeros(1, 16, device="cuda"), 1e-5, None, materialize), w)
        assert calls == [1]
        close(got, x.double() @ w.double().t(), dtype)


def test_fused_qkv_projection_finishes_a_prepared_norm(fusing, twin):
    kernels = fusing
    heads, kv_heads, head_dim, page_size, width = 8, 2, 64, 16, 256
    segments = [(300, 1), (0, 1), (17, 1), (64, 1)]
    _, batch, view = make_paged_case(torch.bfloat16, heads, kv_heads, head_dim, page_size, segments, seed=23)
    g = torch.Generator(device="cuda").manual_seed(24)
    M = len(segments)
    stream = torch.randn(M, width, device="cuda", generator=g) * 2
    norm = _Norm((1.0 + 0.2 * torch.randn(width, device="cuda", generator=g)).to(torch.bfloat16), 1e-5)
    x0 = torch.randn(M, 64, device="cuda", generator=g).to(torch.bfloat16)
    w0 = (torch.randn(width, 64, device="cuda", generator=g) / 8).to(torch.bfloat16)
    prepared = kernels.linear(x0, w0, accumulate=stream, next_norm=norm)
    w = (torch.randn((heads + 2 * kv_heads) * head_dim, width, device="cuda", generator=g) / math.sqrt(width)).to(torch.bfloat16)
    inv_freq = (1.0 / (500000.0 ** (torch.arange(0, head_dim, 2).float() / head_dim))).cuda()
    view2 = SimpleNamespace(keys=view.keys.float(), values=view.values.float(), block_table=view.block_table,
                            page_size=page_size, window=None)
    q = kernels.fused_qkv_rope(prepared, w, batch, inv_freq, head_dim, heads, kv_heads, head_dim, view, True)
    assert q is not None
    qkv = (_rms(stream, norm.weight, 1e-5) @ w.double().t()).float()
    twin.rope_kv_write(qkv, batch, inv_freq, head_dim, heads, kv_heads, head_dim, view2, True)
    close(q, qkv[:, :heads * head_dim], torch.bfloat16)
    close(view.keys, view2.keys, torch.bfloat16)
    close(view.values, view2.values, torch.bfloat16)
    kernels.check_status()
