"""Each part alone against the plain implementation's function for it."""

import pytest
import torch

import helpers
import plain_llama
from tt_transformers_b200.cache import CacheManager
from tt_transformers_b200.parts import PartSpec, Runtime, build_part

pytestmark = pytest.mark.gpu
DTYPES = [(torch.float32, 2e-5), (torch.bfloat16, 3e-2)]


def runtime(dtype):
    from tt_transformers_b200.kernels import load_kernels

    return Runtime(kernels=load_kernels("cuda:0"), device=torch.device("cuda:0"), dtype=dtype)


def close(got, ref, tol):
    assert float((got.float().cpu() - ref).abs().max()) <= tol * max(1.0, float(ref.abs().max()))


@pytest.mark.parametrize("dtype,tol", DTYPES)
def test_rmsnorm_part(dtype, tol):
    g = torch.Generator().manual_seed(0)
    w = 1 + 0.1 * torch.randn(80, generator=g)
    part = build_part("norm", PartSpec("rmsnorm", dict(width=80, eps=1e-6, weight_name="n")))
    assert [(s.name, s.shape) for s in part.tensor_specs()] == [("n", (80,))]
    part.bind({"n": w}, runtime(dtype))
    x, d = torch.randn(9, 80, generator=g), torch.randn(9, 80, generator=g)
    res = x.cuda()
    out = part.forward_add(res, d.cuda().to(dtype))
    close(res, x + d.to(dtype).float(), 1e-6)
    close(out, plain_llama.rms_norm(x + d.to(dtype).float(), w, 1e-6), tol)
    close(part.forward_add(res, None), plain_llama.rms_norm(x + d.to(dtype).float(), w, 1e-6), tol)


@pytest.mark.parametrize("dtype,tol", DTYPES)
def test_swiglu_part(dtype, tol):
    g = torch.Generator().manual_seed(1)
    w = {"f.gate_proj.weight": torch.randn(200, 80, generator=g) * 0.1, "f.up_proj.weight": torch.randn(200, 80, generator=g) * 0.1,
         "f.down_proj.weight": torch.randn(80, 200, generator=g) * 0.1}
    if dtype == torch.bfloat16:
        w = {k: v.to(dtype).float() for k, v in w.items()}
    part = build_part("feed_forward", PartSpec("swiglu", dict(width=80, inter=200, prefix="f.")))
    part.bind(w, runtime(dtype))
    for rows in (1, 7, 40, 100):
        x = torch.randn(rows, 80, generator=g).to(dtype)
        close(part.forward(x.cuda(), None), plain_llama.swiglu(x.float(), w, "f."), tol)


def test_rotary_part_gives_the_plain_frequencies():
    scaling = {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
               "original_max_position_embeddings": 64}
    part = build_part("position", PartSpec("rotary", dict(rotary_dim=32, theta=500000.0, scaling=scaling)))
    part.bind({}, runtime(torch.float32))
    inv_freq, rotary_dim = part.rotation()
    assert rotary_dim == 32 and torch.equal(inv_freq.cpu(), plain_llama.rope_inverse_frequencies(32, 500000.0, scaling))
    assert build_part("position", PartSpec("none")).rotation() is None


@pytest.mark.parametrize("dtype,tol", DTYPES)
@pytest.mark.parametrize("heads,kv_heads,head_dim,window", [(4, 2, 16, None), (3, 1, 32, None), (8, 2, 64, None),
                                                              (6, 2, 128, None), (4, 4, 48, 10), (8, 2, 64, 40)])
def test_attention_part_with_its_cache(dtype, tol, heads, kv_heads, head_dim, window):
    """The mixer alone on the cache manager's pages: portions of two requests, then single
    tokens, against the plain attention block over the whole sequences."""
    from tt_transformers_b200.engine.step import Engine, StepEntry  # noqa: F401  (StepBatch is built by hand below)
    from tt_transformers_b200.parts import StepBatch

    width, page = 72, 8
    g = torch.Generator().manual_seed(2)
    rt = runtime(dtype)
    names = ("q_proj", "k_proj", "v_proj", "o_proj")
    shapes = ((heads * head_dim, width), (kv_heads * head_dim, width), (kv_heads * head_dim, width), (width, heads * head_dim))
    w = {f"a.{n}.weight": (torch.randn(s, generator=g) * 0.1).to(dtype).float() for n, s in zip(names, shapes)}
    position = build_part("position", PartSpec("rotary", dict(rotary_dim=head_dim, theta=10000.0, scaling=None)))
    position.bind({}, rt)
    part = build_part("mixer", PartSpec("attention", dict(width=width, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                                                          prefix="a.", position=position, window=window)))
    part.bind(w, rt)
    cache = CacheManager([part.cache_request()], page, 40, 2, 160, rt.device, dtype)
    for tensor in cache.groups[0].storage.values():
        tensor.fill_(float("nan"))
    xs = {"a": torch.randn(70, width, generator=g).to(dtype), "b": torch.randn(45, width, generator=g).to(dtype)}
    config = {"num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim, "hidden_size": width}
    inv_freq = plain_llama.rope_inverse_frequencies(head_dim, 10000.0, None)

    def plain_block(x):
        T = x.shape[0]
        q = plain_llama.rope_rotate((x @ w["a.q_proj.weight"].T).view(T, heads, head_dim), torch.arange(T), inv_freq)
        k = plain_llama.rope_rotate((x @ w["a.k_proj.weight"].T).view(T, kv_heads, head_dim), torch.arange(T), inv_freq)
        v = (x @ w["a.v_proj.weight"].T).view(T, kv_heads, head_dim)
        return plain_llama.causal_attention(q, k, v, window).reshape(T, -1) @ w["a.o_proj.weight"].T

    ref = {rid: plain_block(x.float()) for rid, x in xs.items()}
    got = {rid: [] for rid in xs}
    done = {"a": 0, "b": 0}
    for rid in xs:
        cache.admit(rid)
    plan = [(("a", 33), ("b", 20)), (("a", 30),), (("b", 24), ("a", 1)), (("a", 1), ("b", 1)), (("a", 5),)]
    for step in plan:
        lens = [n for _, n in step]
        pos0 = [done[r] for r, _ in step]
        for (r, n) in step:
            cache.reserve(r, done[r] + n)
        slots = [cache.slot(r) for r, _ in step]
        T = sum(lens)
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        positions = [p + i for p, n in zip(pos0, lens) for i in range(n)]
        seg_of = [s for s, n in enumerate(lens) for _ in range(n)]
        dev = lambda v: torch.tensor(v, dtype=torch.int32, device=rt.device)  # noqa: E731
        W = max(1, -(-max(p + n for p, n in zip(pos0, lens)) // page))
        batch = StepBatch(num_tokens=T, num_segments=len(step), token_ids=dev([0] * T), positions=dev(positions),
                          seg_of_token=dev(seg_of), cu_seqlens=dev(cu), seg_pos0=dev(pos0), seg_slot=dev(slots),
                          want_rows=dev([0]), num_wanted=0, seg_lens=lens, seg_pos0_list=pos0, seg_slot_list=slots,
                          max_seg_len=max(lens), max_context=max(p + n for p, n in zip(pos0, lens)))
        batch.block_tables[0] = torch.from_numpy(cache.table_rows(0, slots, W).copy()).to(rt.device)
        x = torch.cat([xs[r][done[r]:done[r] + n] for r, n in step]).cuda()
        out = part.forward(x, batch, cache.view(0, batch), True)
        start = 0
        for r, n in step:
            got[r].append(out[start:start + n].float().cpu())
            start += n
            done[r] += n
            cache.commit(r, done[r])
        cache.audit()
    rt.kernels.check_status()
    for rid in xs:
        close(torch.cat(got[rid]), ref[rid], tol)


@pytest.mark.parametrize("dtype,tol", DTYPES)
def test_embedding_and_head_parts(dtype, tol):
    """The `table` embedding with a scale; the `linear` head with a weight of its own and tied to the embedding,
    with a scale and a cap on its logits."""
    g = torch.Generator().manual_seed(5)
    table = (torch.randn(300, 72, generator=g) * 0.3).to(dtype).float()
    own = (torch.randn(300, 72, generator=g) * 0.3).to(dtype).float()
    emb = build_part("embedding", PartSpec("table", dict(vocab=300, width=72, weight_name="e", scale=72 ** 0.5)))
    tied = build_part("head", PartSpec("linear", dict(vocab=300, width=72, weight_name=None, logit_cap=4.0)))
    untied = build_part("head", PartSpec("linear", dict(vocab=300, width=72, weight_name="h", scale=0.25)))
    assert tied.tied and not untied.tied and tied.tensor_specs() == [] and untied.tensor_specs()[0].name == "h"
    tied.tie(emb)
    rt = runtime(dtype)
    for part in (emb, tied, untied):
        part.bind({"e": table, "h": own}, rt)
    assert tied.weight.data_ptr() == emb.table.data_ptr()            # the same storage, not a copy
    ids = torch.tensor([0, 299, 17, 17, 5], dtype=torch.int32, device="cuda")
    close(emb.forward(ids), table[ids.long().cpu()] * 72 ** 0.5, 1e-6)
    h = torch.randn(6, 72, generator=g).to(dtype)
    close(tied.forward(h.cuda()), 4.0 * torch.tanh(h.float() @ table.T / 4.0), tol)
    close(untied.forward(h.cuda()), 0.25 * (h.float() @ own.T), tol)
    with pytest.raises(ValueError):
        build_part("head", PartSpec("linear", dict(vocab=3, width=2, weight_name=None, logit_cap=0.0)))
