"""Benchmarks for the evaluation harness (reference evaluation/benchmarks.py).

Each benchmark builds ``prompts`` (and private ground truths) in its constructor, may
override generation settings through ``generation_overrides``, and scores a list of
generations in ``compute_metrics``. Datasets come from the Hugging Face hub on demand
(``datasets.load_dataset``), exactly as in the reference; scoring rules match it:

* GSM8k: last ``\\boxed{}`` (else the whole text), commas and ``$`` removed, parsed as an int;
* MATH / AIME: ``math_verify`` equivalence of the last ``\\boxed{}`` against the reference;
* DROP: the lm-eval DROP metric (EM / F1) when ``lm_eval`` is installed;
* multiple choice (MMLU, ARC, HellaSwag, Winogrande, BoolQ): one generated token compared
  with the gold letter; an answer outside the option letters counts as invalid and earns
  1 / n_options (chance) credit; MMLU / MMLU-Pro report per-subject and macro averages;
* AIME majority voting: maj@k over the k most frequent valid answers, and unbiased pass@k.
"""
from __future__ import annotations

import re
from collections import Counter, defaultdict
from dataclasses import dataclass
from typing import Any, Callable, Optional

from hrm_text_b200.utils.functions import compute_benchmark_micro_macro_avg, last_boxed_only_string


def _load(*args, **kwargs):
    from datasets import load_dataset
    return load_dataset(*args, **kwargs)


class BaseBenchmark:
    def __init__(self):
        self.prompts: list[str] = []
        self.ground_truths: list[Any] = []

    @property
    def generation_overrides(self) -> dict:
        return {}

    def compute_metrics(self, generations: list[str]) -> dict:
        raise NotImplementedError


def _accuracy(correct: float, invalid: int, n: int) -> dict:
    return {"n": n, "acc": correct / max(1, n), "invalid": invalid / max(1, n)}


# ---------------------------------------------------------------------------------------
# math
# ---------------------------------------------------------------------------------------
def parse_int_answer(text: str) -> Optional[int]:
    boxed = last_boxed_only_string(text)
    if boxed:
        text = boxed
    text = text.replace(",", "").replace("$", "").strip()
    try:
        return int(float(text))
    except (ValueError, OverflowError):
        return None


class GSM8k(BaseBenchmark):
    def __init__(self, split: str = "test"):
        super().__init__()
        ds = _load("gsm8k", "main", split=split)
        self.prompts = list(ds["question"])
        self.ground_truths = [int(a.split("####")[-1].strip().replace(",", "")) for a in ds["answer"]]

    def compute_metrics(self, generations):
        correct = invalid = 0
        for text, gt in zip(generations, self.ground_truths):
            ans = parse_int_answer(text)
            if ans is None:
                invalid += 1
            elif ans == gt:
                correct += 1
        return _accuracy(correct, invalid, len(generations))


class MATH(BaseBenchmark):
    def __init__(self, split: str = "test"):
        super().__init__()
        from datasets import get_dataset_config_names
        for subset in get_dataset_config_names("EleutherAI/hendrycks_math"):
            for item in _load("EleutherAI/hendrycks_math", subset, split=split):
                label = last_boxed_only_string(item["solution"])
                assert label is not None
                self.prompts.append(item["problem"])
                self.ground_truths.append(label)

    def compute_metrics(self, generations):
        from math_verify import parse, verify
        correct = invalid = 0
        for text, gt in zip(generations, self.ground_truths):
            ans = last_boxed_only_string(text)
            if ans is None:
                invalid += 1
                ans = text
            if verify(parse(gt), parse(ans)):
                correct += 1
        return _accuracy(correct, invalid, len(generations))


# ---------------------------------------------------------------------------------------
# reading comprehension
# ---------------------------------------------------------------------------------------
class DROP(BaseBenchmark):
    """Few-shot DROP. Exemplars: the first ``num_shots`` training examples (or ``shots``)."""

    def __init__(self, split: str = "validation", num_shots: int = 3, shots: Optional[list[str]] = None):
        super().__init__()
        from lm_eval.tasks.drop.utils import process_docs
        if shots is None:
            shots = []
            for doc in process_docs(_load("EleutherAI/drop", split="train")):
                shots.append(f"{doc['passage']}\nQ: {doc['question']}\nA: {doc['answers'][0][0]}")
                if len(shots) >= num_shots:
                    break
        prefix = "".join(f"{s}\n\n" for s in shots[:num_shots])
        self.ground_truths = list(process_docs(_load("EleutherAI/drop", split=split)))
        self.prompts = [f"{prefix}{d['passage']}\nQ: {d['question']}\nA:" for d in self.ground_truths]

    def compute_metrics(self, generations):
        from lm_eval.tasks.drop.utils import process_results
        em = f1 = 0.0
        for text, doc in zip(generations, self.ground_truths):
            r = process_results(doc, [text.strip()])
            em += r.get("em", 0.0)
            f1 += r.get("f1", 0.0)
        n = len(generations)
        return {"n": n, "em": em / max(1, n), "f1": f1 / max(1, n)}


# ---------------------------------------------------------------------------------------
# multiple choice
# ---------------------------------------------------------------------------------------
@dataclass
class MCQDoc:
    query: str
    choices: list[str]
    gold_index: int


def format_mcq(doc: MCQDoc, include_gold: bool) -> tuple[str, list[str]]:
    letters = [chr(ord("A") + i) for i in range(len(doc.choices))]
    lines = [doc.query.strip()] + [f"{l}. {c.strip()}" for l, c in zip(letters, doc.choices)]
    answer = f"Answer: {letters[doc.gold_index]}" if include_gold else "Answer:"
    return "\n".join(lines) + "\n" + answer, letters


def mcq_prompt(target: MCQDoc, shots: list[MCQDoc]) -> tuple[str, list[str]]:
    prefix = "".join(format_mcq(s, True)[0] + "\n\n" for s in shots)
    text, letters = format_mcq(target, False)
    return prefix + text, letters


def score_letter(pred: str, valid: set, gold: str) -> tuple[float, bool]:
    """(credit, invalid): invalid answers earn chance-level credit."""
    p = pred.strip().upper()
    if p not in valid:
        return 1.0 / len(valid), True
    return (1.0 if p == gold else 0.0), False


class StandardMCQBenchmark(BaseBenchmark):
    @property
    def generation_overrides(self) -> dict:
        return {"max_tokens": 1}

    def compute_metrics(self, generations):
        correct, invalid = 0.0, 0
        for pred, gt in zip(generations, self.ground_truths):
            credit, bad = score_letter(pred, gt["valid_set"], gt["gold"])
            correct += credit
            invalid += bad
        return _accuracy(correct, invalid, len(generations))


class MMLU(StandardMCQBenchmark):
    def __init__(self, split: str = "test", num_shots: int = 5, special_shots: Optional[dict] = None):
        super().__init__()
        special_shots = special_shots or {}
        shots = defaultdict(list)
        for row in _load("cais/mmlu", "all", split="dev"):
            shots[row["subject"]].append(MCQDoc(row["question"], row["choices"], row["answer"]))
        for row in _load("cais/mmlu", "all", split=split):
            subj = row["subject"]
            doc = MCQDoc(row["question"], row["choices"], row["answer"])
            prompt, letters = mcq_prompt(doc, shots[subj][: special_shots.get(subj, num_shots)])
            self.prompts.append(prompt)
            self.ground_truths.append({"valid_set": set(letters), "gold": letters[doc.gold_index], "subject": subj})

    def compute_metrics(self, generations):
        stats = defaultdict(lambda: {"n": 0, "correct": 0.0, "invalid": 0})
        for pred, gt in zip(generations, self.ground_truths):
            s = stats[gt["subject"]]
            credit, bad = score_letter(pred, gt["valid_set"], gt["gold"])
            s["n"] += 1
            s["correct"] += credit
            s["invalid"] += bad
        return compute_benchmark_micro_macro_avg(stats)


class MMLUPro(BaseBenchmark):
    """Open-ended MMLU-Pro: the last bracketed option letter ``(X)`` (else a bare letter) wins."""

    def __init__(self, split: str = "test"):
        super().__init__()
        for item in _load("TIGER-Lab/MMLU-Pro", "default", split=split):
            letters = [chr(65 + i) for i in range(len(item["options"]))]
            opts = "".join(f"({l}) {o}\n" for l, o in zip(letters, item["options"]))
            self.prompts.append(item["question"] + "\nOptions:\n" + opts)
            self.ground_truths.append((item["answer"], letters, item["category"]))

    @staticmethod
    def extract_letter(text: str, options: list[str]) -> Optional[str]:
        alt = "|".join(options)
        found = re.findall(r"\((" + alt + r")\)", text) or re.findall(r"\b(" + alt + r")\b", text)
        return found[-1] if found else None

    def compute_metrics(self, generations):
        stats = defaultdict(lambda: {"n": 0, "correct": 0.0, "invalid": 0})
        for text, (gold, options, cat) in zip(generations, self.ground_truths):
            boxed = last_boxed_only_string(text)
            ans = self.extract_letter(boxed if boxed else text, options)
            s = stats[cat]
            s["n"] += 1
            if ans is None:
                s["invalid"] += 1
                s["correct"] += 1.0 / len(options)
            elif ans == gold:
                s["correct"] += 1
        return compute_benchmark_micro_macro_avg(stats)


class HFMCQBenchmark(StandardMCQBenchmark):
    """Hub MCQ dataset -> few-shot letter prompts (shots from ``shot_split[:num_shots]``)."""

    def __init__(self, path: str, split: str, shot_split: str, num_shots: int,
                 row_to_doc: Callable[[dict], MCQDoc], name: Optional[str] = None):
        super().__init__()
        docs = [row_to_doc(r) for r in _load(path, name, split=split)]
        shots = [row_to_doc(r) for r in _load(path, name, split=f"{shot_split}[:{num_shots}]")] if num_shots else []
        for doc in docs:
            prompt, letters = mcq_prompt(doc, shots)
            self.prompts.append(prompt)
            self.ground_truths.append({"valid_set": set(letters), "gold": letters[doc.gold_index]})


class ARC(HFMCQBenchmark):
    def __init__(self, split: str = "test", subset: str = "ARC-Challenge", num_shots: int = 25):
        super().__init__("allenai/ai2_arc", split, "validation", num_shots,
                         lambda r: MCQDoc(r["question"], r["choices"]["text"],
                                          r["choices"]["label"].index(r["answerKey"])), name=subset)


class HellaSwag(HFMCQBenchmark):
    def __init__(self, split: str = "validation", num_shots: int = 10):
        super().__init__("Rowan/hellaswag", split, "train", num_shots,
                         lambda r: MCQDoc(f"{r['ctx_a']} {r['ctx_b'].capitalize()}\n"
                                          "Question: Which is the most logical continuation?",
                                          r["endings"], int(r["label"])))


class Winogrande(HFMCQBenchmark):
    def __init__(self, split: str = "validation", num_shots: int = 5):
        super().__init__("allenai/winogrande", split, "train", num_shots,
                         lambda r: MCQDoc(r["sentence"], [r["option1"], r["option2"]], int(r["answer"]) - 1),
                         name="winogrande_debiased")


class BoolQ(HFMCQBenchmark):
    def __init__(self, split: str = "validation", num_shots: int = 5):
        super().__init__("google/boolq", split, "train", num_shots,
                         lambda r: MCQDoc(f"{r['passage']}\nQuestion: {r['question'].capitalize()}?",
                                          ["Yes", "No"], 0 if r["answer"] else 1))


# ---------------------------------------------------------------------------------------
# majority voting
# ---------------------------------------------------------------------------------------
def unbiased_pass_at_k(n: int, c: int, k: int) -> float:
    """1 - C(n-c, k) / C(n, k): probability that k of n samples (c correct) include a correct one."""
    if n - c < k:
        return 1.0
    fail = 1.0
    for j in range(k):
        fail *= (n - c - j) / (n - j)
    return 1.0 - fail


class AIMEMajorityVoting(BaseBenchmark):
    def __init__(self, year: str = "25", n: int = 256, pass_k: tuple = (1, 10, 100)):
        super().__init__()
        self.n, self.pass_k = n, list(pass_k)
        for item in _load(f"math-ai/aime{year}", split="test"):
            gt = item.get("answer")
            if gt is None and item.get("solution"):
                gt = last_boxed_only_string(item["solution"])
            self.prompts.extend([item["problem"]] * n)
            self.ground_truths.append(int(gt))

    def compute_metrics(self, generations):
        from math_verify import parse, verify
        maj = {k: 0 for k in self.pass_k}
        pas = {k: 0.0 for k in self.pass_k}
        out = {}
        for i, gt in enumerate(self.ground_truths):
            votes, c = [], 0
            for text in generations[i * self.n:(i + 1) * self.n]:
                boxed = last_boxed_only_string(text)
                text = boxed if boxed is not None else text
                c += bool(verify(str(gt), parse(text)))
                try:
                    v = int(text)
                    if 1 <= v <= 999:
                        votes.append(v)
                except ValueError:
                    pass
            ranked = Counter(votes).most_common()
            out[f"{i}_valid"] = len(votes)
            out[f"{i}_cons_count"] = ranked[0][1] if ranked else 0
            for k in self.pass_k:
                if gt in [a for a, _ in ranked[:k]]:
                    maj[k] += 1
                if self.n >= k:
                    pas[k] += unbiased_pass_at_k(self.n, c, k)
        total = max(1, len(self.ground_truths))
        out |= {f"maj_pass@{k}": v / total for k, v in maj.items()}
        out |= {f"pass@{k}": v / total for k, v in pas.items()}
        return out
