"""The framework takes parts and architectures it has never seen, without a change to its files:
a toy mixer with a running state of its own, a layer order that names a layer twice and lets a
layer read another layer's cache, and layers with and without a window side by side."""

from dataclasses import dataclass

import pytest
import torch

import helpers
import plain_llama
from tt_transformers_b200 import register_architecture, register_part
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.engine.step import build_engine
from tt_transformers_b200.parts import (Block, CacheRequest, LayerCall, LayerSpec, Mixer, ModelSpec, PartSpec, SlotState,
                                        TensorSpec)
from tt_transformers_b200.weights import write_model_folder

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------------------- a toy mixer with state
class RunningMeanMixer(Mixer):
    """y_t = W * mean(x_0 .. x_t). Its state per request: the running sum (width numbers); the
    count is the position. Defined here, in the test, with plain torch operations."""

    def __init__(self, width, weight_name, position=None):
        self.width, self.weight_name = width, weight_name

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.width, self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = runtime.matrix(tensors[self.weight_name])

    def cache_request(self):
        return SlotState((self.width,))

    def forward(self, x, batch, cache, write_cache=True):
        out = torch.empty_like(x)
        start = 0
        for n, pos0, slot in zip(batch.seg_lens, batch.seg_pos0_list, cache.slot_list):
            sums = cache.state[slot] + torch.cumsum(x[start:start + n].float(), dim=0)
            counts = torch.arange(pos0 + 1, pos0 + n + 1, device=x.device, dtype=torch.float32)[:, None]
            out[start:start + n] = ((sums / counts).to(x.dtype) @ self.weight.t())
            if write_cache:
                cache.state[slot] = sums[-1]
            start += n
        return out


@dataclass(frozen=True)
class ToyConfig:
    width: int
    layers: int
    vocab: int
    inter: int
    eps: float


def toy_load_config(d):
    return ToyConfig(d["width"], d["layers"], d["vocab"], d["inter"], d["eps"])


def toy_model_spec(cfg):
    layers = tuple(LayerSpec(
        norm1=PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.eps, weight_name=f"toy.{i}.norm1")),
        mixer=PartSpec("running_mean", dict(width=cfg.width, weight_name=f"toy.{i}.mix")),
        norm2=PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.eps, weight_name=f"toy.{i}.norm2")),
        feed_forward=PartSpec("swiglu", dict(width=cfg.width, inter=cfg.inter, prefix=f"toy.{i}.ff.")),
    ) for i in range(cfg.layers))
    return ModelSpec(vocab_size=cfg.vocab, width=cfg.width, embedding=PartSpec("table", dict(vocab=cfg.vocab, width=cfg.width, weight_name="toy.embed")), layers=layers,
                     order=tuple(LayerCall(i) for i in range(cfg.layers)),
                     final_norm=PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.eps, weight_name="toy.norm")),
                     head=PartSpec("linear", dict(vocab=cfg.vocab, width=cfg.width, weight_name="toy.head")))


def toy_plain_forward(cfg, w, tokens):
    x = w["toy.embed"][torch.as_tensor(tokens)]
    counts = torch.arange(1, len(tokens) + 1, dtype=torch.float32)[:, None]
    for i in range(cfg["layers"]):
        h = plain_llama.rms_norm(x, w[f"toy.{i}.norm1"], cfg["eps"])
        x = x + (torch.cumsum(h, 0) / counts) @ w[f"toy.{i}.mix"].T
        h = plain_llama.rms_norm(x, w[f"toy.{i}.norm2"], cfg["eps"])
        x = x + plain_llama.swiglu(h, w, f"toy.{i}.ff.")
    return plain_llama.rms_norm(x, w["toy.norm"], cfg["eps"]) @ w["toy.head"].T


def test_a_toy_mixer_with_state_is_registered_built_and_stepped(tmp_path):
    register_part("mixer", "running_mean", RunningMeanMixer)
    register_architecture("ToyRunningMeanForTests", toy_load_config, toy_model_spec)
    cfg = {"architectures": ["ToyRunningMeanForTests"], "width": 48, "layers": 2, "vocab": 100, "inter": 72, "eps": 1e-5}
    folder = write_model_folder(str(tmp_path / "toy"), cfg, seed=5, std=0.2, norm_std=0.1, dtype=torch.float32)
    _, w = plain_llama.read_model_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(100, n, i) for i, n in enumerate((9, 30, 17, 5, 22))}
    ref = {rid: toy_plain_forward(cfg, w, toks) for rid, toks in requests.items()}
    for dtype, tol in (("float32", 1e-4), ("bfloat16", 5e-2)):
        engine = build_engine(folder, EngineConfig(dtype=dtype, max_batch_size=4, max_seq_len=64, device="cuda:0"))
        assert engine.graphs is None                      # a mixer that reads host lists is never captured
        assert [type(g.request).__name__ for g in engine.cache.groups] == ["SlotState"]
        for steps in (helpers.steps_whole(requests), helpers.steps_portions(requests), helpers.steps_mixed(requests)):
            got = helpers.run_steps(engine, steps)
            for rid in ref:
                assert helpers.relative_error(got[rid], ref[rid]) < tol, (dtype, rid)
        assert engine.cache.free_slots == 4
        engine.close()


# ---------------------------------------------------------------------------- layer order as data; windows
@dataclass(frozen=True)
class OrderConfig:
    width: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float
    theta: float
    windows: tuple          # per layer: None or a window
    order: tuple            # (layer, cache_of or None)


def order_load_config(d):
    return OrderConfig(d["width"], d["heads"], d["kv_heads"], d["head_dim"], d["inter"], d["vocab"], d["eps"],
                       d["theta"], tuple(d["windows"]), tuple(tuple(o) for o in d["order"]))


def order_model_spec(cfg):
    rotary = PartSpec("rotary", dict(rotary_dim=cfg.head_dim, theta=cfg.theta, scaling=None))
    layers = tuple(LayerSpec(
        norm1=PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.eps, weight_name=f"l.{i}.n1")),
        mixer=PartSpec("attention", dict(width=cfg.width, heads=cfg.heads, kv_heads=cfg.kv_heads,
                                         head_dim=cfg.head_dim, prefix=f"l.{i}.attn.", window=window)),
        position=rotary,
        norm2=PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.eps, weight_name=f"l.{i}.n2")),
        feed_forward=PartSpec("swiglu", dict(width=cfg.width, inter=cfg.inter, prefix=f"l.{i}.ff.")),
    ) for i, window in enumerate(cfg.windows))
    return ModelSpec(vocab_size=cfg.vocab, width=cfg.width, embedding=PartSpec("table", dict(vocab=cfg.vocab, width=cfg.width, weight_name="emb")), layers=layers,
                     order=tuple(LayerCall(l, c) for l, c in cfg.order),
                     final_norm=PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.eps, weight_name="norm")),
                     head=PartSpec("linear", dict(vocab=cfg.vocab, width=cfg.width, weight_name=None)))


def order_plain_forward(cfg, w, tokens):
    """Whole sequence, no cache: the layer order run by hand with the plain parts."""
    T = len(tokens)
    H, G, hd = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    positions = torch.arange(T)
    inv_freq = plain_llama.rope_inverse_frequencies(hd, cfg["theta"], None)
    x = w["emb"][torch.as_tensor(tokens)]
    kept = {}
    for entry, (layer, cache_of) in enumerate(cfg["order"]):
        p = f"l.{layer}."
        h = plain_llama.rms_norm(x, w[p + "n1"], cfg["eps"])
        q = plain_llama.rope_rotate((h @ w[p + "attn.q_proj.weight"].T).view(T, H, hd), positions, inv_freq)
        if cache_of is None:
            k = plain_llama.rope_rotate((h @ w[p + "attn.k_proj.weight"].T).view(T, G, hd), positions, inv_freq)
            v = (h @ w[p + "attn.v_proj.weight"].T).view(T, G, hd)
            kept[entry] = (k, v)
        else:
            k, v = kept[cache_of]
        o = plain_llama.causal_attention(q, k, v, cfg["windows"][layer]).reshape(T, H * hd)
        x = x + o @ w[p + "attn.o_proj.weight"].T
        h = plain_llama.rms_norm(x, w[p + "n2"], cfg["eps"])
        x = x + plain_llama.swiglu(h, w, p + "ff.")
    return plain_llama.rms_norm(x, w["norm"], cfg["eps"]) @ w["emb"].T


@pytest.mark.parametrize("head_dim", [32, 64])
def test_layer_order_shared_caches_and_windows(tmp_path, head_dim):
    register_architecture("OrderForTests", order_load_config, order_model_spec)
    cfg = {"architectures": ["OrderForTests"], "width": 96, "heads": 4, "kv_heads": 2, "head_dim": head_dim,
           "inter": 160, "vocab": 200, "eps": 1e-5, "theta": 10000.0,
           "windows": [None, 24, None],
           # layer 0 runs twice with caches of its own, layer 2 reads the cache of the first entry,
           # layer 1 keeps a window of 24 keys
           "order": [[0, None], [1, None], [0, None], [2, 0], [1, None]]}
    folder = write_model_folder(str(tmp_path / "order"), cfg, seed=9, std=0.08, norm_std=0.1, dtype=torch.float32)
    _, w = plain_llama.read_model_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(200, n, 20 + i) for i, n in enumerate((70, 33, 120, 9, 64))}
    ref = {rid: order_plain_forward(cfg, w, toks) for rid, toks in requests.items()}
    for dtype, tol in (("float32", 1e-4), ("bfloat16", 5e-2)):
        for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
            steps = make_steps(requests)
            pages = -(-helpers.max_live_tokens(requests, steps, rounding=8) // 8)
            engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=8, num_pages=pages, max_batch_size=4,
                                                       max_seq_len=128, device="cuda:0"))
            kinds = [(type(g.request).__name__, g.request.window, len(g.units)) for g in engine.cache.groups]
            assert kinds == [("PagedKV", None, 2), ("PagedKV", 24, 2)]       # entry 3 owns no unit: it reads entry 0's
            for g in engine.cache.groups:
                for tensor in g.storage.values():
                    tensor.fill_(float("nan"))       # a read of a slot that was never written would show
            got = helpers.run_steps(engine, steps)
            engine.cache.audit()
            for rid in ref:
                assert helpers.relative_error(got[rid], ref[rid]) < tol, (dtype, make_steps.__name__, rid)
            engine.close()


def test_windowed_pages_come_back_while_the_request_lives(tmp_path):
    register_architecture("OrderForTests", order_load_config, order_model_spec)
    cfg = {"architectures": ["OrderForTests"], "width": 64, "heads": 2, "kv_heads": 1, "head_dim": 32, "inter": 96,
           "vocab": 100, "eps": 1e-5, "theta": 10000.0, "windows": [16], "order": [[0, None]]}
    folder = write_model_folder(str(tmp_path / "win"), cfg, seed=3, std=0.1, dtype=torch.float32)
    _, w = plain_llama.read_model_folder(folder)
    tokens = helpers.random_tokens(100, 200, 1)
    ref = order_plain_forward(cfg, w, tokens)
    # 200 tokens would need 50 pages of 4; the window of 16 never holds more than 6 (+ the step's own)
    engine = build_engine(folder, EngineConfig(dtype="float32", page_size=4, num_pages=12, max_batch_size=1,
                                               max_seq_len=256, device="cuda:0"))
    steps = helpers.steps_portions({"a": tokens}, sizes=(7, 5, 3, 2, 2, 11, 4, 2, 16, 9))
    got = helpers.run_steps(engine, steps)
    assert helpers.relative_error(got["a"], ref) < 1e-4
    assert engine.cache.free_pages() == 12


# ---------------------------------------------------------------------------- a routed feed-forward and a learned position encoding
class ToyRoutedFF:
    """Top-1 routing over small SwiGLU experts: router logits and their softmax in float32, the chosen
    expert's output scaled by its probability. Plain torch operations, defined in the test."""

    def __init__(self, width, inter, experts, prefix):
        self.width, self.inter, self.experts, self.prefix = width, inter, experts, prefix

    def tensor_specs(self):
        p = self.prefix
        return ([TensorSpec(p + "router", (self.experts, self.width))]
                + [TensorSpec(f"{p}{e}.{n}", s) for e in range(self.experts)
                   for n, s in (("gate", (self.inter, self.width)), ("up", (self.inter, self.width)),
                                ("down", (self.width, self.inter)))])

    def bind(self, tensors, runtime):
        self.runtime = runtime
        p = self.prefix
        self.router = tensors[p + "router"].to(runtime.device, torch.float32)
        self.w = [{n: runtime.matrix(tensors[f"{p}{e}.{n}"]) for n in ("gate", "up", "down")} for e in range(self.experts)]

    def forward(self, x, batch):
        probs = torch.softmax(x.float() @ self.router.t(), dim=-1)
        weight, choice = probs.max(dim=-1)
        out = torch.zeros_like(x)
        k = self.runtime.kernels
        for e in range(self.experts):
            rows = (choice == e).nonzero().flatten()
            if rows.numel():
                xe = x[rows].contiguous()
                gate_up = torch.cat([self.w[e]["gate"], self.w[e]["up"]], 0)
                ye = k.linear(k.linear_swiglu(xe, gate_up), self.w[e]["down"])     # the engine's own kernels per expert
                out[rows] = (ye.float() * weight[rows, None]).to(x.dtype)
        return out


class LearnedPositions:
    """An absolute encoding: a learned table row is added to every embedded token; nothing is rotated."""

    def __init__(self, width, max_positions, weight_name):
        self.width, self.max_positions, self.weight_name = width, max_positions, weight_name

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.max_positions, self.width))]

    def bind(self, tensors, runtime):
        self.table = tensors[self.weight_name].to(runtime.device, torch.float32)

    def embed(self, x, batch):
        return x + self.table[batch.positions.long()]

    def rotation(self):
        return None


def routed_model_spec(cfg):
    layers = tuple(LayerSpec(
        norm1=PartSpec("rmsnorm", dict(width=cfg["width"], eps=1e-5, weight_name=f"m.{i}.n1")),
        mixer=PartSpec("attention", dict(width=cfg["width"], heads=2, kv_heads=1, head_dim=32, prefix=f"m.{i}.attn.")),
        norm2=PartSpec("rmsnorm", dict(width=cfg["width"], eps=1e-5, weight_name=f"m.{i}.n2")),
        feed_forward=PartSpec("toy_routed", dict(width=cfg["width"], inter=cfg["inter"], experts=cfg["experts"],
                                                 prefix=f"m.{i}.moe.")),
    ) for i in range(cfg["layers"]))
    return ModelSpec(vocab_size=cfg["vocab"], width=cfg["width"],
                     embedding=PartSpec("table", dict(vocab=cfg["vocab"], width=cfg["width"], weight_name="emb")), layers=layers,
                     order=tuple(LayerCall(i) for i in range(cfg["layers"])),
                     final_norm=PartSpec("rmsnorm", dict(width=cfg["width"], eps=1e-5, weight_name="norm")),
                     head=PartSpec("linear", dict(vocab=cfg["vocab"], width=cfg["width"], weight_name="head")),
                     input_position=PartSpec("toy_learned", dict(width=cfg["width"], max_positions=cfg["positions"],
                                                                 weight_name="pos")))


def routed_plain_forward(cfg, w, tokens):
    T = len(tokens)
    x = w["emb"][torch.as_tensor(tokens)] + w["pos"][:T]
    for i in range(cfg["layers"]):
        p = f"m.{i}."
        h = plain_llama.rms_norm(x, w[p + "n1"], 1e-5)
        q = (h @ w[p + "attn.q_proj.weight"].T).view(T, 2, 32)            # no rotation: order comes from the table
        k = (h @ w[p + "attn.k_proj.weight"].T).view(T, 1, 32)
        v = (h @ w[p + "attn.v_proj.weight"].T).view(T, 1, 32)
        x = x + plain_llama.causal_attention(q, k, v).reshape(T, 64) @ w[p + "attn.o_proj.weight"].T
        h = plain_llama.rms_norm(x, w[p + "n2"], 1e-5)
        probs = torch.softmax(h @ w[p + "moe.router"].T, dim=-1)
        weight, choice = probs.max(dim=-1)
        out = torch.zeros_like(h)
        for t in range(T):
            e = int(choice[t])
            ws = {"gate_proj.weight": w[f"{p}moe.{e}.gate"], "up_proj.weight": w[f"{p}moe.{e}.up"],
                  "down_proj.weight": w[f"{p}moe.{e}.down"]}
            out[t] = plain_llama.swiglu(h[t:t + 1], ws, "")[0] * weight[t]
        x = x + out
    return plain_llama.rms_norm(x, w["norm"], 1e-5) @ w["head"].T


def test_a_routed_feed_forward_and_a_learned_position_encoding(tmp_path):
    register_part("feed_forward", "toy_routed", ToyRoutedFF)
    register_part("position", "toy_learned", LearnedPositions)
    register_architecture("ToyRoutedForTests", lambda d: d, routed_model_spec)
    cfg = {"architectures": ["ToyRoutedForTests"], "width": 64, "layers": 2, "vocab": 120, "inter": 96, "experts": 3,
           "positions": 128}
    folder = write_model_folder(str(tmp_path / "routed"), cfg, seed=11, std=0.15, norm_std=0.1, dtype=torch.float32)
    _, w = plain_llama.read_model_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(120, n, 40 + i) for i, n in enumerate((50, 21, 37, 8))}
    ref = {rid: routed_plain_forward(cfg, w, toks) for rid, toks in requests.items()}
    engine = build_engine(folder, EngineConfig(dtype="float32", page_size=8, max_batch_size=4, max_seq_len=128, device="cuda:0"))
    assert engine.graphs is None                           # a part that does not declare itself safe to capture
    for steps in (helpers.steps_whole(requests), helpers.steps_decode_tail(requests, 8), helpers.steps_mixed(requests)):
        got = helpers.run_steps(engine, steps)
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 1e-4, rid


# ---------------------------------------------------------------------------- a whole toy architecture out of kinds the package has not
@dataclass(frozen=True)
class LatentPages(CacheRequest):
    """One tensor per token instead of keys and values: a latent vector, from which the mixer makes both.
    A page holds page_size latents."""

    latent: int
    window: object = None
    paged = True

    def storage(self, page_size):
        return {"latent": ((page_size, self.latent), None)}

    def view(self, tensors, *, block_table, page_size, **_):
        return {"latent": tensors["latent"], "block_table": block_table, "page_size": page_size}


class LatentAttention(Mixer):
    """Single-head causal attention whose cache holds c_t = Wc h_t only; keys Wk c and values Wv c are made
    from the cached latents of the request at every step. Plain torch operations."""

    def __init__(self, width, latent, prefix, position=None):
        self.width, self.latent, self.prefix = width, latent, prefix

    def tensor_specs(self):
        p = self.prefix
        return [TensorSpec(p + "q", (self.latent, self.width)), TensorSpec(p + "c", (self.latent, self.width)),
                TensorSpec(p + "k", (self.latent, self.latent)), TensorSpec(p + "v", (self.width, self.latent))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.w = {n: runtime.matrix(tensors[self.prefix + n]) for n in "qckv"}

    def cache_request(self):
        return LatentPages(self.latent)

    def forward(self, x, batch, cache, write_cache=True):
        P, pages, table = cache["page_size"], cache["latent"], cache["block_table"]
        c = (x.float() @ self.w["c"].float().t()).to(x.dtype)
        if write_cache:
            pos = batch.positions.long()
            pages[table[batch.seg_of_token.long(), pos // P].long(), pos % P] = c
        q = x.float() @ self.w["q"].float().t()
        out = torch.empty_like(x)
        start = 0
        for r, (n, pos0) in enumerate(zip(batch.seg_lens, batch.seg_pos0_list)):
            ctx = pos0 + n
            held = pages[table[r, :-(-ctx // P)].long()].reshape(-1, self.latent)[:ctx].float()
            keys, values = held @ self.w["k"].float().t(), held @ self.w["v"].float().t()
            scores = q[start:start + n] @ keys.t() * self.latent ** -0.5
            visible = torch.arange(ctx, device=x.device)[None, :] <= torch.arange(pos0, ctx, device=x.device)[:, None]
            probs = torch.softmax(scores.masked_fill(~visible, float("-inf")), dim=-1)
            out[start:start + n] = (probs @ values).to(x.dtype)
            start += n
        return out


class SandwichBlock(Block):
    """Norms before AND after each sub-layer: x += post1(mixer(norm1(x))); x += post2(ff(norm2(x)))."""

    slots = {"norm1": "norm", "mixer": "mixer", "post1": "norm", "norm2": "norm", "feed_forward": "feed_forward",
             "post2": "norm"}

    def __init__(self, norm1, mixer, post1, norm2, feed_forward, post2):
        self.norm1, self.mixer, self.post1 = norm1, mixer, post1
        self.norm2, self.feed_forward, self.post2 = norm2, feed_forward, post2

    def forward(self, x, delta, batch, cache, write_cache=True):
        h = self.norm1.forward_add(x, delta)
        mixed = self.post1.forward_add(self.mixer.forward(h, batch, cache, write_cache).float(), None)
        h = self.norm2.forward_add(x, mixed)
        return x, self.post2.forward_add(self.feed_forward.forward(h, batch).float(), None)


def latent_model_spec(cfg):
    W, V = cfg["width"], cfg["vocab"]
    norm = lambda name: PartSpec("rmsnorm", dict(width=W, eps=cfg["eps"], weight_name=name))  # noqa: E731
    layers = tuple(LayerSpec(
        block="toy_sandwich",
        norm1=norm(f"t.{i}.n1"), mixer=PartSpec("toy_latent", dict(width=W, latent=cfg["latent"], prefix=f"t.{i}.mix.")),
        post1=norm(f"t.{i}.p1"), norm2=norm(f"t.{i}.n2"),
        feed_forward=PartSpec("swiglu", dict(width=W, inter=cfg["inter"], prefix=f"t.{i}.ff.")), post2=norm(f"t.{i}.p2"),
    ) for i in range(cfg["layers"]))
    return ModelSpec(vocab_size=V, width=W,
                     embedding=PartSpec("table", dict(vocab=V, width=W, weight_name="emb", scale=cfg["embed_scale"])),
                     layers=layers, order=tuple(LayerCall(i) for i in range(cfg["layers"])), final_norm=norm("norm"),
                     head=PartSpec("linear", dict(vocab=V, width=W, weight_name=None, logit_cap=cfg["logit_cap"])))


def latent_plain_forward(cfg, w, tokens, layers=None):
    T, L = len(tokens), cfg["latent"]
    x = w["emb"][torch.as_tensor(tokens)] * cfg["embed_scale"]
    visible = torch.arange(T)[None, :] <= torch.arange(T)[:, None]
    for i in range(cfg["layers"] if layers is None else layers):
        p = f"t.{i}."
        h = plain_llama.rms_norm(x, w[p + "n1"], cfg["eps"])
        c = h @ w[p + "mix.c"].T
        scores = (h @ w[p + "mix.q"].T) @ (c @ w[p + "mix.k"].T).T * L ** -0.5
        mixed = torch.softmax(scores.masked_fill(~visible, float("-inf")), dim=-1) @ (c @ w[p + "mix.v"].T)
        x = x + plain_llama.rms_norm(mixed, w[p + "p1"], cfg["eps"])
        h = plain_llama.rms_norm(x, w[p + "n2"], cfg["eps"])
        x = x + plain_llama.rms_norm(plain_llama.swiglu(h, w, p + "ff."), w[p + "p2"], cfg["eps"])
    logits = plain_llama.rms_norm(x, w["norm"], cfg["eps"]) @ w["emb"].T
    return cfg["logit_cap"] * torch.tanh(logits / cfg["logit_cap"])


def test_a_toy_architecture_with_scaled_embedding_capped_head_post_norms_and_a_latent_cache(tmp_path):
    """Nothing under the package changes for: an embedding with a scale, a head with a cap on its logits, a block
    kind with six parts, and a cache request that stores one tensor per token."""
    register_part("mixer", "toy_latent", LatentAttention)
    register_part("block", "toy_sandwich", SandwichBlock)
    register_architecture("ToyLatentForTests", lambda d: d, latent_model_spec)
    cfg = {"architectures": ["ToyLatentForTests"], "width": 56, "layers": 3, "vocab": 150, "inter": 88, "latent": 24,
           "eps": 1e-5, "embed_scale": 56 ** 0.5, "logit_cap": 6.0}
    folder = write_model_folder(str(tmp_path / "latent"), cfg, seed=21, std=0.15, norm_std=0.1, dtype=torch.float32)
    _, w = plain_llama.read_model_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(150, n, 60 + i) for i, n in enumerate((61, 18, 40, 7, 33))}
    ref = {rid: latent_plain_forward(cfg, w, toks) for rid, toks in requests.items()}
    assert max(float(r.abs().max()) for r in ref.values()) > 3.0          # the cap bends these logits (tanh(0.5) = 0.46)
    for dtype, tol in (("float32", 1e-4), ("bfloat16", 5e-2)):
        for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
            steps = make_steps(requests)
            pages = -(-helpers.max_live_tokens(requests, steps, rounding=8) // 8)
            engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=8, num_pages=pages, max_batch_size=4,
                                                       max_seq_len=64, device="cuda:0"))
            (group,) = engine.cache.groups
            assert list(group.storage) == ["latent"] and group.storage["latent"].shape == (3, pages + 1, 8, 24)
            group.storage["latent"].fill_(float("nan"))
            got = helpers.run_steps(engine, steps)
            engine.cache.audit()
            assert engine.cache.free_pages() == pages
            for rid in ref:
                assert helpers.relative_error(got[rid], ref[rid]) < tol, (dtype, make_steps.__name__, rid)
            engine.close()
    # the model cut to its first two layer-order entries, through the ModelSpec (no architecture-specific code)
    engine = build_engine(folder, EngineConfig(dtype="float32", page_size=8, max_batch_size=2, max_seq_len=64,
                                               device="cuda:0"), n_layers=2)
    got = helpers.run_steps(engine, helpers.steps_whole({"r1": requests["r1"]}))
    assert helpers.relative_error(got["r1"], latent_plain_forward(cfg, w, requests["r1"], layers=2)) < 1e-4
    engine.close()
