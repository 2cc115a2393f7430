"""Generate a continuation of one prompt and print it.

The options are the reference demo's: --prompt, --hf-model, --max-new-tokens (40),
--max-seq-len (2048) (examples/llama32_1b/demo.py:38-44). --hf-model is a model folder on
disk (config.json + safetensors); with a tokenizer in the folder the prompt is text and goes
through the chat template, as in the reference; without one the prompt is a list of token
ids ("5,17,3") and token ids are printed. --random NAME runs a named model with random weights.
"""

from __future__ import annotations

import argparse
import os
import sys


def run(llm, prompt, *, max_new_tokens=40, do_sample=False, temperature=1.0, top_k=50, top_p=1.0, seed=None):
    if llm.tokenizer is not None:
        messages = [{"role": "user", "content": prompt}]
        inputs = llm.tokenizer.apply_chat_template(messages, add_generation_prompt=True, tokenize=True,
                                                   return_dict=True, return_tensors="pt")
        outputs = llm.generate(inputs["input_ids"], inputs.get("attention_mask"), max_new_tokens=max_new_tokens,
                               do_sample=do_sample, temperature=temperature, top_k=top_k, top_p=top_p, seed=seed)
        continuation = outputs[:, inputs["input_ids"].shape[1]:]
        return llm.tokenizer.batch_decode(continuation, skip_special_tokens=True)[0]
    try:
        ids = [int(t) for t in prompt.replace(",", " ").split()]
    except ValueError:
        raise SystemExit("the model folder has no tokenizer: give --prompt as token ids, e.g. --prompt '5,17,3'")
    out = llm.generate([ids], max_new_tokens=max_new_tokens, do_sample=do_sample, temperature=temperature,
                       top_k=top_k, top_p=top_p, seed=seed)[0]
    return " ".join(str(t) for t in out)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--prompt", default="Explain paged attention briefly.")
    parser.add_argument("--hf-model", default=None, help="model folder (default: $HF_MODEL)")
    parser.add_argument("--max-new-tokens", type=int, default=40)
    parser.add_argument("--max-seq-len", type=int, default=2048)
    parser.add_argument("--random", default=None, help="run a named model with random weights instead of --hf-model")
    parser.add_argument("--dtype", default="bfloat16", choices=("bfloat16", "float32"))
    parser.add_argument("--do-sample", action="store_true")
    parser.add_argument("--temperature", type=float, default=1.0)
    parser.add_argument("--top-k", type=int, default=50)
    parser.add_argument("--top-p", type=float, default=1.0)
    parser.add_argument("--seed", type=int, default=None)
    args = parser.parse_args(argv)
    from .common import load

    hf_model = args.hf_model or (None if args.random else os.environ.get("HF_MODEL"))
    if not hf_model and not args.random:
        parser.error("give --hf-model DIR (or set HF_MODEL), or --random NAME")
    llm = load(hf_model, args.random, max_batch_size=1, max_seq_len=args.max_seq_len, dtype=args.dtype)
    try:
        print(run(llm, args.prompt, max_new_tokens=args.max_new_tokens, do_sample=args.do_sample,
                  temperature=args.temperature, top_k=args.top_k, top_p=args.top_p, seed=args.seed))
    finally:
        llm.cleanup()


if __name__ == "__main__":
    main()
