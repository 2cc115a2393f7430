"""Shared helpers of the tests: prompts, ways of cutting requests into steps, comparison."""

from __future__ import annotations

import torch

import plain_llama


def random_tokens(vocab, count, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (count,), generator=g).tolist()


def relative_error(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / max |ref|."""
    return float((got.float().cpu() - ref.float().cpu()).abs().max() / ref.float().abs().max())


def plain_logits(folder, requests):
    """{id: logits [len, vocab]} of whole sequences by the plain implementation."""
    config, weights = plain_llama.read_model_folder(folder)
    return {rid: plain_llama.forward(config, weights, toks) for rid, toks in requests.items()}


# ---------------------------------------------------------------------------- ways of cutting
def steps_whole(requests):
    """Each request alone and whole, one after the other."""
    steps = []
    for rid, toks in requests.items():
        steps.append({"entries": [{"id": rid, "tokens": toks, "want": list(range(len(toks)))}], "end": [rid]})
    return steps


def steps_decode_tail(requests, tail=32):
    """Most of a request in one step, its last `tail` tokens one by one."""
    steps = []
    for rid, toks in requests.items():
        head = max(1, len(toks) - tail)
        steps.append({"entries": [{"id": rid, "tokens": toks[:head], "want": list(range(head))}],
                      "end": [rid] if head == len(toks) else []})
        for i in range(head, len(toks)):
            steps.append({"entries": [{"id": rid, "tokens": [toks[i]], "want": [0]}],
                          "end": [rid] if i == len(toks) - 1 else []})
    return steps


def steps_portions(requests, sizes=(7, 5, 3, 2, 2, 11, 4, 2, 16, 9)):
    """Each request alone in portions of changing size, down to two tokens."""
    steps = []
    for rid, toks in requests.items():
        i, k = 0, 0
        while i < len(toks):
            n = min(sizes[k % len(sizes)], len(toks) - i)
            steps.append({"entries": [{"id": rid, "tokens": toks[i:i + n], "want": list(range(n))}],
                          "end": [rid] if i + n == len(toks) else []})
            i, k = i + n, k + 1
    return steps


def steps_mixed(requests, max_live=4, seed=0, decode_tail=8):
    """Up to max_live requests at a time: portions of some beside single tokens of others.
    A request runs its first part in portions and its last `decode_tail` tokens one by one;
    when one ends, the next starts, so that its pages are used again."""
    g = torch.Generator().manual_seed(seed)
    waiting = list(requests.items())
    live = {}      # id -> next index
    steps = []
    while waiting or live:
        while waiting and len(live) < max_live:
            rid, _ = waiting.pop(0)
            live[rid] = 0
        entries, end = [], []
        for rid in list(live):
            toks = requests[rid]
            i = live[rid]
            if int(torch.randint(0, 5, (1,), generator=g)) == 0 and len(live) > 1:
                continue                       # this request sits the step out
            if i >= len(toks) - decode_tail:
                n = 1
            else:
                n = min(int(torch.randint(2, 12, (1,), generator=g)), len(toks) - decode_tail - i)
                n = max(n, 1)
            entries.append({"id": rid, "tokens": toks[i:i + n], "want": list(range(n))})
            live[rid] = i + n
            if i + n == len(toks):
                end.append(rid)
                del live[rid]
        if entries:
            steps.append({"entries": entries, "end": end})
    return steps


def max_live_tokens(requests, steps, rounding=64):
    """The most tokens that live requests hold at any time, each rounded up to `rounding`."""
    held, peak = {}, 0
    for s in steps:
        for e in s["entries"]:
            held[e["id"]] = held.get(e["id"], 0) + len(e["tokens"])
        peak = max(peak, sum(-(-n // rounding) * rounding for n in held.values()))
        for rid in s["end"]:
            del held[rid]
    return peak


def run_steps(engine, steps):
    """Drive engine.step with the steps; {id: logits [len, vocab]} of everything wanted."""
    from tt_transformers_b200.engine.step import StepEntry

    got = {}
    for s in steps:
        entries = [StepEntry(e["id"], e["tokens"], e["want"]) for e in s["entries"]]
        logits = engine.step(entries).float().cpu()
        row = 0
        for e in s["entries"]:
            for _ in e["want"]:
                got.setdefault(e["id"], []).append(logits[row])
                row += 1
        for rid in s["end"]:
            engine.finish(rid)
    engine.kernels.check_status()
    return {rid: torch.stack(rows) for rid, rows in got.items()}


def steps_many(requests, live, tail=44, seed=0, portion=(2, 40)):
    """Many requests at a time: up to `live` are live; each runs its prompt part in portions beside the others'
    decoded tokens and its last `tail` tokens one by one; nobody sits a step out, so that between admissions the
    steps hold one token per request (the shape that is captured and replayed). When a request ends, the next
    waiting one is admitted in the following step and takes over its pages."""
    g = torch.Generator().manual_seed(seed)
    waiting = list(requests)
    at = {}
    steps = []
    while waiting or at:
        while waiting and len(at) < live:
            at[waiting.pop(0)] = 0
        entries, end = [], []
        for rid in list(at):
            toks, i = requests[rid], at[rid]
            head = max(1, len(toks) - tail)
            if i >= head:
                n = 1
            else:
                n = min(int(torch.randint(portion[0], portion[1] + 1, (1,), generator=g)), head - i)
            entries.append({"id": rid, "tokens": toks[i:i + n], "want": [n - 1] if i + n >= head else []})
            at[rid] = i + n
            if at[rid] == len(toks):
                end.append(rid)
                del at[rid]
        steps.append({"entries": entries, "end": end})
    return steps


def wanted_positions(steps):
    """{id: [positions]} of the logits that run_steps collects for these steps, in order."""
    at, out = {}, {}
    for s in steps:
        for e in s["entries"]:
            base = at.get(e["id"], 0)
            out.setdefault(e["id"], []).extend(base + w for w in e["want"])
            at[e["id"]] = base + len(e["tokens"])
    return out


def error_stats(got, ref, margin=0.02):
    """Over all requests: the largest and the mean |got - ref| relative to the largest |ref|, how often the best
    token agrees, and how often it agrees on rows whose reference leads its runner-up by more than `margin`
    times the largest |ref| (rows that rounding should not flip)."""
    worst = mean = 0.0
    rows = agree = clear = clear_agree = 0
    for rid in ref:
        g, r = got[rid].float().cpu(), ref[rid].float().cpu()
        scale = float(r.abs().max())
        diff = (g - r).abs()
        worst = max(worst, float(diff.max()) / scale)
        mean += float(diff.mean(dim=-1).sum()) / scale
        same = g.argmax(-1) == r.argmax(-1)
        top2 = r.topk(2, dim=-1).values
        lead = (top2[:, 0] - top2[:, 1]) > margin * scale
        rows += r.shape[0]
        agree += int(same.sum())
        clear += int(lead.sum())
        clear_agree += int((same & lead).sum())
    return {"max": worst, "mean": mean / rows, "top1": agree / rows, "clear_rows": clear,
            "clear_top1": clear_agree / max(clear, 1)}
