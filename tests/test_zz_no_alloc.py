"""The entry point for callers that cannot allocate device memory (csrc/no_alloc.h).

Some hosts of the kernel library run under a memory plan that is not theirs to change: a
serving process whose pool belongs to another component, code inside a graph capture, a GPU
whose memory is handed out in full. For them the library has one decode-attention entry point
whose scratch memory is a fixed array in the library image. This test calls it through its
exported C symbol, as such a host would, and compares its output with the ordinary entry
point's (which takes scratch memory from the caller; the results must be the same bits) and with
plain PyTorch attention, on two calls in a row of which the first is the larger: the second call
finds the first call's leftovers in the array and must not be disturbed by them.

The file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def make_case(segments, heads, kv_heads, head_dim, page_size, contexts, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    pages_needed = sum(-(-(c + 1) // page_size) for c in contexts)
    qkv = torch.randn(segments, (heads + 2 * kv_heads) * head_dim, device="cuda", generator=g).to(torch.bfloat16)
    keys = torch.randn(pages_needed + 1, kv_heads, page_size, head_dim, device="cuda", generator=g).to(torch.bfloat16)
    values = torch.randn(pages_needed + 1, kv_heads, page_size, head_dim, device="cuda", generator=g).to(torch.bfloat16)
    width = max(-(-(c + 1) // page_size) for c in contexts)
    table = torch.zeros(segments, width, dtype=torch.int32)
    order = (torch.randperm(pages_needed, generator=torch.Generator().manual_seed(seed)) + 1).tolist()
    for r, c in enumerate(contexts):
        for i in range(-(-(c + 1) // page_size)):
            table[r, i] = order.pop()
    cu = torch.arange(segments + 1, dtype=torch.int32, device="cuda")
    pos0 = torch.tensor(contexts, dtype=torch.int32, device="cuda")
    return qkv, keys, values, table.cuda(), cu, pos0


def run_both(lib, heads, kv_heads, head_dim, page_size, contexts, splits, seed):
    """One call of the entry point that allocates nothing and one of the ordinary entry point (scratch memory from
    the caller) on the same inputs; also what plain PyTorch gives for them."""
    from types import SimpleNamespace

    from torch_kernels import TorchKernels

    segments = len(contexts)
    scale = head_dim ** -0.5
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    qkv, keys, values, table, cu, pos0 = make_case(segments, heads, kv_heads, head_dim, page_size, contexts, seed)
    out = torch.full((segments, heads * head_dim), float("nan"), dtype=torch.bfloat16, device="cuda")
    code = lib.ttb_paged_attention_decode_noalloc(
        ptr(qkv), qkv.stride(0), ptr(out), ptr(cu), ptr(pos0), ptr(keys), ptr(values), ptr(table), table.shape[1],
        page_size, segments, heads, kv_heads, head_dim, ctypes.c_float(scale), 0, splits, stream)
    assert code == 0
    ref = torch.empty_like(out)
    partial_o = torch.empty(segments * heads * splits * head_dim, dtype=torch.float32, device="cuda")
    partial_ml = torch.empty(segments * heads * splits * 2, dtype=torch.float32, device="cuda")
    code = lib.ttb_paged_attention_mma(ptr(qkv), qkv.stride(0), ptr(ref), ptr(cu), ptr(pos0), ptr(keys),
                                       ptr(values), ptr(table), table.shape[1], page_size, None, None, segments,
                                       segments, heads, kv_heads, head_dim, ctypes.c_float(scale), 0, 1, splits,
                                       ptr(partial_o), ptr(partial_ml), stream)
    assert code == 0
    torch.cuda.synchronize()
    batch = SimpleNamespace(seg_lens=[1] * segments, seg_pos0_list=list(contexts))
    view = SimpleNamespace(keys=keys.float(), values=values.float(), block_table=table, page_size=page_size, window=None)
    plain = TorchKernels("cuda").paged_attention(qkv.float(), batch, heads, kv_heads, head_dim, scale, view)
    return out, ref, plain


# Two calls in a row per case, the first LARGER than the second (more requests, more key splits, or the other
# head size): the second call finds the first call's partial results all over the part of the array it uses, and
# beyond it.
@pytest.mark.parametrize("first,second", [
    ((8, 2, 64, 16, [700, 3, 129, 2048, 90, 1500], 8), (8, 2, 64, 16, [700, 3, 129, 2048], 6)),
    ((8, 2, 64, 16, [2048, 1, 333], 7), (6, 2, 128, 8, [64, 999], 4)),
    ((6, 2, 128, 8, [999, 64, 500], 5), (8, 2, 64, 16, [15, 16, 17], 2)),
])
def test_no_alloc_entry_point_matches_the_ordinary_one(first, second):
    from tt_transformers_b200.kernels import load_kernels

    lib = load_kernels("cuda:0").lib
    lib.ttb_paged_attention_decode_noalloc.restype = ctypes.c_int          # the exported C symbol
    lib.ttb_noalloc_scratch_bytes.restype = ctypes.c_uint
    assert lib.ttb_noalloc_scratch_bytes() == 16 << 20
    for call, case in enumerate((first, second)):
        out, ref, plain = run_both(lib, *case, seed=call)
        assert not torch.isnan(out.float()).any()
        # the same kernels with the same key splits, only the scratch memory lies elsewhere: the same bits
        assert torch.equal(out, ref), (call, float((out.float() - ref.float()).abs().max()))
        # and not only against itself: plain PyTorch attention over the same pages (tolerance of the kernel tests)
        err = float((out.float() - plain.float()).abs().max())
        assert err <= 2e-2 * max(1.0, float(plain.float().abs().max())), (call, err)


def test_no_alloc_entry_point_refuses_what_exceeds_its_scratch():
    from tt_transformers_b200.kernels import load_kernels

    lib = load_kernels("cuda:0").lib
    lib.ttb_paged_attention_decode_noalloc.restype = ctypes.c_int
    # 4096 requests x 32 heads x 16 splits x (64 + 2) floats = 528 MiB: far beyond 16 MiB; refused before any pointer is read
    code = lib.ttb_paged_attention_decode_noalloc(None, 0, None, None, None, None, None, None, 1, 16, 4096, 32, 8, 64,
                                                  ctypes.c_float(0.125), 0, 16, None)
    assert code == -4
