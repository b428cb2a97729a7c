"""Prepare SFT data in the training data layout (same CLI as the reference's script).

    python scripts/prepare_sft_data.py --train my_sft.jsonl --tokenizer tokenizer.json \
        --output /dev/shm/sft_data --epochs 10

Input JSONL rows: ``{"instruction": ..., "response": ..., "condition": "direct"}`` (condition
optional). Each sample becomes ``<boq><condition token>instruction<eoq>`` (the prefix) and
``response<eoa>`` (the supervised part). Samples whose response tokenises to nothing are
dropped (a packed batch of only such samples has no response tokens at all).

Output: ``metadata.json``, ``tokens.npy``, ``tokenizer_info.json``, a copy of the tokenizer,
and one shuffled index set per epoch (``epoch_{e}/{inst,resp}_{start,len}.npy``, Philox
permutations from ``--seed``).
"""
from __future__ import annotations

import argparse
import json
import shutil
from pathlib import Path

import numpy as np

DEFAULT_CONDITIONS = "direct=<|object_ref_start|>,cot=<|object_ref_end|>,noisy=<|quad_start|>,synth=<|quad_end|>"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--train", required=True)
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--epochs", type=int, required=True)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--context-size", type=int, default=4097)
    ap.add_argument("--boq", default="<|im_start|>")
    ap.add_argument("--eoq", default="<|im_end|>")
    ap.add_argument("--eoa", default="<|box_end|>")
    ap.add_argument("--conditions", default=DEFAULT_CONDITIONS)
    args = ap.parse_args(argv)

    from tokenizers import Tokenizer
    out = Path(args.output)
    out.mkdir(parents=True, exist_ok=True)
    tok = Tokenizer.from_file(args.tokenizer)

    def token_id(name: str) -> int:
        tid = tok.token_to_id(name)
        if tid is None:
            raise ValueError(f"special token {name!r} not in tokenizer vocab")
        return tid

    boq, eoq, eoa = token_id(args.boq), token_id(args.eoq), token_id(args.eoa)
    cond_ids, cond_tokens = {}, {}
    for pair in args.conditions.split(","):
        key, name = pair.split("=")
        cond_ids[key], cond_tokens[key] = token_id(name), name

    rows = [json.loads(line) for line in open(args.train, encoding="utf-8") if line.strip()]
    print(f"Loaded {len(rows)} samples from {args.train}")
    tokens: list[int] = []
    inst_start, inst_len, resp_start, resp_len = [], [], [], []
    skipped = 0
    for row in rows:
        cond = row.get("condition", "direct")
        if cond not in cond_ids:
            raise ValueError(f"sample condition {cond!r} not in --conditions map (known: {sorted(cond_ids)})")
        inst = tok.encode(row["instruction"], add_special_tokens=False).ids
        resp = tok.encode(row["response"], add_special_tokens=False).ids
        if not resp:
            skipped += 1
            continue
        s = len(tokens)
        tokens += [boq, cond_ids[cond], *inst, eoq]
        inst_start.append(s)
        inst_len.append(len(tokens) - s)
        s = len(tokens)
        tokens += [*resp, eoa]
        resp_start.append(s)
        resp_len.append(len(tokens) - s)
    if skipped:
        print(f"Skipped {skipped} samples with empty response")
    if not inst_start:
        raise ValueError("no samples left after filtering")

    lens = np.array(inst_len, dtype=np.int64) + np.array(resp_len, dtype=np.int64)
    if int(lens.max()) >= args.context_size:
        raise ValueError(f"longest sample is {int(lens.max())} tokens but --context-size is {args.context_size}; "
                         "bump --context-size.")
    print(f"Tokens: {len(tokens):,}  avg sample = {lens.mean():.1f}  max = {int(lens.max())}")
    np.save(out / "tokens.npy", np.array(tokens, dtype=np.int32))
    if Path(args.tokenizer).resolve() != (out / "tokenizer.json").resolve():
        shutil.copyfile(args.tokenizer, out / "tokenizer.json")
    info = {"tokenizer_path": str(out), "boq": args.boq, "eoq": args.eoq, "eoa": args.eoa,
            "condition_mapping": cond_tokens, "vocab_size": tok.get_vocab_size(with_added_tokens=True)}
    (out / "tokenizer_info.json").write_text(json.dumps(info))
    # vocab_size stays null in metadata: the loader derives the padded vocabulary itself.
    meta = {"tokenizer_info": info, "vocab_size": None, "max_seq_len": args.context_size,
            "total_length": int(lens.sum())}
    (out / "metadata.json").write_text(json.dumps(meta))
    arrays = {k: np.array(v, dtype=np.int64) for k, v in
              (("inst_start", inst_start), ("inst_len", inst_len), ("resp_start", resp_start), ("resp_len", resp_len))}
    rng = np.random.Generator(np.random.Philox(seed=args.seed))
    for e in range(args.epochs):
        perm = rng.permutation(len(inst_start))
        d = out / f"epoch_{e}"
        d.mkdir(exist_ok=True)
        for name, arr in arrays.items():
            np.save(d / f"{name}.npy", arr[perm])
    print(f"Wrote {args.epochs} epoch shuffles to {out}")
    print(f"Done. Point cfg.data.path to: {out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
