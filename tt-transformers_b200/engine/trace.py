"""Trace replay: given token ids go through the model step by step and logits are written.

It samples nothing and has no forward pass of its own: every step is one call of the
engine's step function, on the engine's own cache and kernels. Its ancestors in the
reference are the teacher-forcing loops, which feed ground-truth tokens and record the
prediction (examples/common/run_helpers.py:201-289; qualification/readiness/teacher_forcing.py:30-181).

Input: one JSON object per line,
    {"step": 0, "entries": [{"id": "a", "tokens": [5, 17, 3], "want": [0, 2]}], "end": []}
For a step that wants logits, <out>/<step>.f32 holds them as little-endian float32
[wanted, vocab], in the order of the entries and of `want`. After every step a line
`done <step>` is printed and flushed.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

from ..config.engine import EngineConfig
from .step import StepEntry, build_engine

MAX_LIVE = 4            # requests live at a time in a trace
REQUEST_ROUNDING = 64   # each request's token count is rounded up to this for --max-tokens


def run_trace(model: str, dtype: str, out_dir: str, max_tokens: int, lines, log=sys.stdout, device="cuda:0",
              kernels=None, page_size: int = 16, cuda_graph: bool = True) -> int:
    """Replay the steps that `lines` yields. Returns the number of steps run. Steps that bring one token
    per request run as generation runs them: as replays of a captured step (cuda_graph False: eagerly)."""
    os.makedirs(out_dir, exist_ok=True)
    if REQUEST_ROUNDING % page_size:
        raise ValueError(f"page_size {page_size} must divide {REQUEST_ROUNDING}")
    num_pages = max(1, -(-max_tokens // page_size))
    config = EngineConfig(dtype=dtype, page_size=page_size, num_pages=num_pages, max_batch_size=MAX_LIVE,
                          max_seq_len=max(max_tokens, page_size), max_step_tokens=max(max_tokens, 1) * MAX_LIVE,
                          max_chunk_tokens=max(max_tokens, 1), cuda_graph=cuda_graph, device=device)
    engine = build_engine(model, config, kernels=kernels)
    steps = 0
    for line in lines:
        line = line.strip()
        if not line:
            continue
        record = json.loads(line)
        step = record["step"]
        entries = [StepEntry(e["id"], e["tokens"], e.get("want", [])) for e in record.get("entries", [])]
        logits = engine.step(entries)
        if logits.shape[0] > 0:
            data = logits.detach().to("cpu").numpy().astype("<f4", copy=False)
            path = os.path.join(out_dir, f"{step}.f32")
            with open(path + ".tmp", "wb") as f:
                f.write(np.ascontiguousarray(data).tobytes())
            os.replace(path + ".tmp", path)
        engine.kernels.check_status()
        for rid in record.get("end", []):
            engine.finish(rid)
        steps += 1
        print(f"done {step}", file=log, flush=True)
    engine.close()
    return steps
