"""Evaluation harness: grouping by generation config, scoring rules, helpers."""
import evaluation.benchmarks as B
from evaluation.main import EvaluationConfig, run
from hrm_text_b200.utils.functions import compute_benchmark_micro_macro_avg, last_boxed_only_string


class _Toy(B.BaseBenchmark):
    def __init__(self, answers=(1, 2, 3)):
        super().__init__()
        self.prompts = [f"q{a}" for a in answers]
        self.ground_truths = list(answers)

    def compute_metrics(self, generations):
        ok = sum(B.parse_int_answer(g) == gt for g, gt in zip(generations, self.ground_truths))
        return {"n": len(generations), "acc": ok / len(generations)}


class _ToyMCQ(B.StandardMCQBenchmark):
    def __init__(self):
        super().__init__()
        doc = B.MCQDoc("2+2?", ["3", "4"], 1)
        prompt, letters = B.mcq_prompt(doc, [B.MCQDoc("1+1?", ["2", "5"], 0)])
        self.prompts = [prompt, prompt]
        self.ground_truths = [{"valid_set": set(letters), "gold": "B"}] * 2


class _Engine:
    def __init__(self):
        self.calls = []

    def generate(self, prompts, **gen):
        self.calls.append((len(prompts), gen))
        return [("\\boxed{" + p[1:] + "}") if p.startswith("q") else "B" for p in prompts]


def test_harness_groups_and_scores(monkeypatch):
    monkeypatch.setattr(B, "Toy", _Toy, raising=False)
    monkeypatch.setattr(B, "ToyMCQ", _ToyMCQ, raising=False)
    cfg = EvaluationConfig(engine="unused", generation_config={"temperature": 0.0},
                           benchmarks=[{"name": "Toy"}, {"name": "Toy", "answers": [5]}, {"name": "ToyMCQ"}])
    eng = _Engine()
    res = run(cfg, engine=eng)
    assert res["Toy"]["acc"] == 1.0 and res["ToyMCQ"]["acc"] == 1.0
    assert len(eng.calls) == 2  # the two Toy instances share one generation batch; MCQ adds max_tokens=1
    assert any(gen.get("max_tokens") == 1 for _, gen in eng.calls)


def test_scoring_helpers():
    assert last_boxed_only_string("a \\boxed{1} b \\boxed{\\frac{1}{2}} c") == "\\frac{1}{2}"
    assert last_boxed_only_string("no box") is None and last_boxed_only_string("\\boxed{open") is None
    assert B.parse_int_answer("so \\boxed{1,200}") == 1200 and B.parse_int_answer("x") is None
    assert B.score_letter(" b ", {"A", "B"}, "B") == (1.0, False)
    assert B.score_letter("Z", {"A", "B", "C", "D"}, "B") == (0.25, True)
    assert B.MMLUPro.extract_letter("I think (B) or maybe (C)", ["A", "B", "C"]) == "C"
    assert B.MMLUPro.extract_letter("answer is A", ["A", "B"]) == "A"
    assert abs(B.unbiased_pass_at_k(10, 3, 1) - 0.3) < 1e-9 and B.unbiased_pass_at_k(5, 4, 2) == 1.0
    avg = compute_benchmark_micro_macro_avg({"x": {"n": 2, "correct": 1, "invalid": 0},
                                             "y": {"n": 4, "correct": 4, "invalid": 1}})
    assert avg["acc"] == 0.75 and avg["n"] == 2 and avg["invalid_y"] == 0.25
