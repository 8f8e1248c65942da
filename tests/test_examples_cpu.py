"""The SFT, DPO and evaluation entry points run end to end on CPU on local files."""

from __future__ import annotations

import csv
import json
import math
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _jsonl(path, rows):
    with open(path, "w") as f:
        f.writelines(json.dumps(r) + "\n" for r in rows)
    return str(path)


def test_run_sft_dpo_and_eval_entry_points(tmp_path):
    from examples.run_dpo import main as dpo_main
    from examples.run_eval import main as eval_main
    from examples.run_sft import main as sft_main

    logs = ["logger.log_dir=" + str(tmp_path / "logs"), "logger.stdout=false"]
    sft = _jsonl(tmp_path / "sft.jsonl", [{"messages": [{"role": "user", "content": f"{i}+1?"},
                                                        {"role": "assistant", "content": str(i + 1)}]}
                                          for i in range(16)])
    state = sft_main(["--config", os.path.join(ROOT, "examples", "configs", "sft_tiny_cpu.yaml"), *logs,
                      "~data.num_prompts", "~data.min_prompt_len", "~data.max_prompt_len",
                      "+data.train.dataset_name=openai_format", f"+data.train.data_path={sft}",
                      "+data.train.processor=sft_processor"])
    assert state["current_step"] == 2

    pref = _jsonl(tmp_path / "pref.jsonl", [{"prompt": f"p{i}", "chosen": "good", "rejected": "bad"}
                                            for i in range(8)])
    state = dpo_main(["--config", os.path.join(ROOT, "examples", "configs", "dpo_tiny_cpu.yaml"), *logs,
                      "~data.num_prompts", "~data.min_prompt_len", "~data.max_prompt_len",
                      "+data.train.dataset_name=BinaryPreferenceDataset", f"+data.train.data_path={pref}"])
    assert state["current_step"] == 2

    with open(tmp_path / "math_500_test.csv", "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["Question", "Answer"])
        w.writerows([[f"{i}+{i}?", str(2 * i)] for i in range(4)])
    res = eval_main(["--config", os.path.join(ROOT, "examples", "configs", "eval_tiny_cpu.yaml"), *logs,
                     "~data.num_prompts", "~data.min_prompt_len", "~data.max_prompt_len", "~env.synthetic",
                     "++data.dataset_name=math500", f"++data.data_path={tmp_path / 'math_500_test.csv'}"])
    assert any(math.isfinite(float(v)) for v in res.values() if isinstance(v, (int, float)))
