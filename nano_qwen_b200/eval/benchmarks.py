"""Benchmark suite runner (reference: eval/benchmarks.py:18-104).

Loads JSONL benchmark files ({"prompt", "choices", "answer"} for multiple
choice, {"prompt", "answer"} for generative) and dispatches to the Evaluator.
The standard definitions point at ``benchmarks/*.jsonl`` like the reference's;
those files are not shipped (no network), so missing files yield empty runs
with a warning, as in the reference.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Dict, List, Optional

from .evaluate import Evaluator

STANDARD_BENCHMARKS = {
    "mmlu": {"type": "multiple_choice", "data_path": "benchmarks/mmlu.jsonl"},
    "arc_challenge": {"type": "multiple_choice", "data_path": "benchmarks/arc_challenge.jsonl"},
    "hellaswag": {"type": "multiple_choice", "data_path": "benchmarks/hellaswag.jsonl"},
    "gsm8k": {"type": "generative", "data_path": "benchmarks/gsm8k.jsonl"},
    "math": {"type": "generative", "data_path": "benchmarks/math.jsonl"},
    "humaneval": {"type": "generative", "data_path": "benchmarks/humaneval.jsonl"},
}


class BenchmarkRunner:
    def __init__(self, evaluator: Evaluator):
        self.evaluator = evaluator
        self.results: Dict[str, dict] = {}

    def run_benchmark(self, name: str, data_path: str, benchmark_type: str = "multiple_choice",
                      max_samples: Optional[int] = None) -> dict:
        qs = self._load_data(data_path, max_samples)
        if benchmark_type == "multiple_choice":
            res = self.evaluator.eval_multiple_choice(qs)
        elif benchmark_type == "generative":
            res = self.evaluator.eval_generative(qs)
        else:
            raise ValueError(f"Unknown benchmark type: {benchmark_type}")
        self.results[name] = res
        print(f"[{name}] accuracy={res['accuracy']:.4f} ({res['correct']}/{res['total']})")
        return res

    def run_all(self, benchmarks: Dict[str, dict]) -> Dict[str, dict]:
        for name, cfg in benchmarks.items():
            self.run_benchmark(name, cfg["data_path"], cfg.get("type", "multiple_choice"),
                               cfg.get("max_samples"))
        return self.results

    def save_results(self, output_path: str) -> None:
        with open(output_path, "w") as f:
            json.dump(self.results, f, indent=2)

    @staticmethod
    def _load_data(path: str, max_samples: Optional[int] = None) -> List[dict]:
        p = Path(path)
        if not p.exists():
            print(f"Warning: benchmark data not found at {path}")
            return []
        out = []
        with open(p) as f:
            for line in f:
                line = line.strip()
                if line:
                    out.append(json.loads(line))
                    if max_samples and len(out) >= max_samples:
                        break
        return out
