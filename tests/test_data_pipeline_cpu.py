"""Data pipeline: tokenizer / chat templates, task processors, response datasets
from local files, ``setup_response_data`` and a GRPO run on a JSONL math set
through ``examples/run_grpo.py`` (CPU)."""

from __future__ import annotations

import json
import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _math_rows(n=24):
    return [{"problem": f"What is {i} + {i + 1}?", "expected_answer": str(2 * i + 1)} for i in range(n)]


def _write_jsonl(path, rows):
    with open(path, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
    return str(path)


def test_byte_tokenizer_and_templates():
    from rl_b200.data.tokenizer import get_tokenizer

    tok = get_tokenizer({"name": "byte"})
    msgs = [{"role": "system", "content": "Be brief."}, {"role": "user", "content": "Hi"}]
    text = tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True)
    assert text == "<|system|>\nBe brief.\n<|user|>\nHi\n<|assistant|>\n"
    ids = tok(text, return_tensors="pt")["input_ids"][0]
    assert tok.decode(ids) == text and int(ids.max()) < tok.vocab_size
    # chat_template: null -> passthrough; a custom template string
    assert get_tokenizer({"name": "byte", "chat_template": None}).apply_chat_template(msgs, tokenize=False) == \
        "Be brief.Hi"
    custom = get_tokenizer({"name": "byte", "chat_template": "{% for m in messages %}[{{ m['content'] }}]{% endfor %}"})
    assert custom.apply_chat_template(msgs, tokenize=False) == "[Be brief.][Hi]"


def test_format_message_log_attributes_every_token():
    from rl_b200.data.processors import format_message_log
    from rl_b200.data.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    conv = [{"role": "user", "content": "2+2?"}, {"role": "assistant", "content": "4"},
            {"role": "user", "content": "and 3+3?"}, {"role": "assistant", "content": "6"}]
    log = format_message_log(conv, tok)
    assert [m["role"] for m in log] == ["user", "assistant", "user", "assistant"]
    flat = torch.cat([m["token_ids"] for m in log])
    whole = tok.encode(tok.apply_chat_template(conv, tokenize=False))
    assert flat.tolist() == [tok.bos_token_id] + whole + [tok.eos_token_id]
    assert tok.decode(log[1]["token_ids"]) == "<|assistant|>\n4\n"


def test_math_processors_prompt_file_and_length_mask(tmp_path):
    from rl_b200.data.processors import TaskDataSpec, math_data_processor, math_hf_data_processor
    from rl_b200.data.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    pf = tmp_path / "prompt.txt"
    pf.write_text("Solve: {}\nPut the answer in \\boxed{{}}.")
    sf = tmp_path / "sys.txt"
    sf.write_text("You are a math tutor.")
    spec = TaskDataSpec("math", prompt_file=str(pf), system_prompt_file=str(sf))
    d = math_hf_data_processor({"messages": [{"role": "user", "content": "1+1"},
                                             {"role": "assistant", "content": "2"}], "task_name": "m"},
                               spec, tok, 4096, 7)
    text = tok.decode(d["message_log"][0]["token_ids"])
    assert "You are a math tutor." in text and "Solve: 1+1\nPut the answer in \\boxed{}." in text
    assert text.endswith("<|assistant|>\n")
    assert d["extra_env_info"] == {"ground_truth": "2"} and d["idx"] == 7 and d["task_name"] == "m"
    assert d["loss_multiplier"] == 1.0 and d["length"] == len(d["message_log"][0]["token_ids"])
    # too long: kept, cut to min(4, max_len // n_messages) tokens, masked
    short = math_data_processor({"problem": "x" * 100, "expected_answer": 3}, TaskDataSpec(), tok, 20, 0)
    assert short["loss_multiplier"] == 0.0 and len(short["message_log"][0]["token_ids"]) == 4
    assert short["extra_env_info"]["ground_truth"] == "3"


def test_load_rows_local_formats(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq

    from rl_b200.data.response_datasets import load_rows

    rows = _math_rows(5)
    jl = _write_jsonl(tmp_path / "a.jsonl", rows)
    js = tmp_path / "a.json"
    js.write_text(json.dumps(rows))
    cols = tmp_path / "c.json"
    cols.write_text(json.dumps({"problem": [r["problem"] for r in rows],
                                "expected_answer": [r["expected_answer"] for r in rows]}))
    pqp = tmp_path / "a.parquet"
    pq.write_table(pa.Table.from_pylist(rows), pqp)
    csvp = tmp_path / "a.csv"
    csvp.write_text("problem,expected_answer\n" + "\n".join(f"{r['problem']},{r['expected_answer']}" for r in rows))
    for p in (jl, js, cols, pqp, csvp):
        got = load_rows(str(p))
        assert len(got) == 5 and got[3] == rows[3], p


def test_named_datasets_from_local_files(tmp_path):
    from rl_b200.data.response_datasets import load_response_dataset

    # GSM8K raw schema: the answer follows "####"
    gsm = _write_jsonl(tmp_path / "gsm.jsonl", [{"question": "q1", "answer": "work... #### 42"},
                                                {"question": "q2", "answer": "#### 7"}])
    ds = load_response_dataset({"dataset_name": "GSM8K", "data_path": gsm})
    assert ds.task_name == "gsm8k" and ds.dataset[0]["messages"][1]["content"] == "42"
    # OpenMathInstruct-2 raw schema with a 25 % validation split
    omi = _write_jsonl(tmp_path / "omi.jsonl", _math_rows(20))
    ds = load_response_dataset({"dataset_name": "OpenMathInstruct-2", "data_path": omi,
                                "split_validation_size": 0.25, "seed": 3})
    assert len(ds.dataset) == 15 and len(ds.val_dataset) == 5
    seen = {r["messages"][0]["content"] for r in ds.dataset} | {r["messages"][0]["content"] for r in ds.val_dataset}
    assert len(seen) == 20
    # NuminaMath keeps only verifiable, validated rows
    num = _write_jsonl(tmp_path / "num.jsonl", [
        {"problem": "a", "answer": "3", "question_type": "math-word-problem", "problem_is_valid": "Yes",
         "solution_is_valid": "Yes"},
        {"problem": "b", "answer": "proof", "question_type": "math-word-problem", "problem_is_valid": "Yes",
         "solution_is_valid": "Yes"},
        {"problem": "c", "answer": "5", "question_type": "proof", "problem_is_valid": "Yes",
         "solution_is_valid": "Yes"},
        {"problem": "d", "answer": "5", "question_type": "math-word-problem", "problem_is_valid": "No",
         "solution_is_valid": "Yes"}])
    ds = load_response_dataset({"dataset_name": "NuminaMath-1.5", "data_path": num})
    assert [r["messages"][0]["content"] for r in ds.dataset] == ["a"]
    # DAPO verl-style rows, AIME with repetition, generic ResponseDataset with custom keys
    dapo = _write_jsonl(tmp_path / "dapo.jsonl", [{"prompt": [{"role": "user", "content": "p"}],
                                                   "reward_model": {"ground_truth": "9"}}])
    assert load_response_dataset({"dataset_name": "DAPOMath17K", "data_path": dapo}).dataset[0]["messages"][1][
        "content"] == "9"
    aime = _write_jsonl(tmp_path / "aime.jsonl", [{"problem": "x", "answer": 12}])
    ds = load_response_dataset({"dataset_name": "AIME2024", "data_path": aime, "repeat": 3})
    assert len(ds.dataset) == 3 and ds.dataset[2]["messages"][1]["content"] == "12" and ds.task_name == "AIME2024"
    os.makedirs(tmp_path / "mine")
    gen = _write_jsonl(tmp_path / "mine" / "set.jsonl", [{"q": "hello", "a": "world"}])
    ds = load_response_dataset({"dataset_name": "ResponseDataset", "data_path": gen, "input_key": "q",
                                "output_key": "a"})
    assert ds.task_name == "mine-set" and ds.dataset[0]["messages"][0]["content"] == "hello"
    with pytest.raises(ValueError):
        load_response_dataset({"dataset_name": "NoSuchDataset"})


def test_nemogym_oasst_arrow_text_and_conversation_datasets(tmp_path):
    import gzip

    from rl_b200.data.processors import PROCESSOR_REGISTRY, TaskDataSpec
    from rl_b200.data.response_datasets import load_response_dataset
    from rl_b200.data.tokenizer import get_tokenizer

    # NeMo-Gym: raw JSONL lines kept as strings, task name from the path, repeat; the processor parses them
    os.makedirs(tmp_path / "gym")
    gym = _write_jsonl(tmp_path / "gym" / "tasks.jsonl", [{"responses_create_params": {"input": "x"},
                                                           "agent_ref": {"name": "a1"}}, {"agent_ref": {"name": "a2"}}])
    ds = load_response_dataset({"dataset_name": "NemoGymDataset", "data_path": gym, "repeat": 2})
    assert ds.task_name == "gym-tasks" and len(ds.dataset) == 4
    assert isinstance(ds.dataset[0]["extra_env_info"], str) and ds.dataset[3]["task_name"] == "gym-tasks"
    d = PROCESSOR_REGISTRY["nemo_gym_data_processor"](ds.dataset[1], None, None, 128, 1)
    assert d["extra_env_info"]["agent_ref"]["name"] == "a2" and d["length"] == 0
    assert d["message_log"][0]["token_ids"].numel() == 0 and d["loss_multiplier"] == 1.0
    # a parquet / json file with a ``text`` column stands in for extra_env_info
    import pyarrow as pa
    import pyarrow.parquet as pq

    txt = str(tmp_path / "gym" / "rows.parquet")
    pq.write_table(pa.table({"text": [json.dumps({"k": 1})]}), txt)
    assert json.loads(load_response_dataset({"dataset_name": "NemoGymDataset", "data_path": txt}).dataset[0][
        "extra_env_info"]) == {"k": 1}
    with pytest.raises(ValueError):
        load_response_dataset({"dataset_name": "NemoGymDataset",
                               "data_path": _write_jsonl(tmp_path / "bad.json", [{"other": 1}, {"other": 2}])})

    # OASST: every root-to-leaf thread, system prompt first, single-turn threads dropped
    tree = {"prompt": {"role": "prompter", "text": "hi", "replies": [
        {"role": "assistant", "text": "A1", "replies": [{"role": "prompter", "text": "more", "replies": []}]},
        {"role": "assistant", "text": "A2", "replies": []}]}}
    lone = {"prompt": {"role": "prompter", "text": "alone", "replies": []}}
    gz = tmp_path / "trees.jsonl.gz"
    with gzip.open(gz, "wt", encoding="utf-8") as f:
        f.write(json.dumps(tree) + "\n" + json.dumps(lone) + "\n")
    ds = load_response_dataset({"dataset_name": "open_assistant", "data_path": str(gz), "split_validation_size": 0})
    threads = [[(m["role"], m["content"]) for m in r["messages"][1:]] for r in ds.dataset]
    assert threads == [[("user", "hi"), ("assistant", "A1"), ("user", "more")], [("user", "hi"), ("assistant", "A2")]]
    assert ds.dataset[0]["messages"][0]["role"] == "system" and ds.task_name == "oasst"

    # arrow_text: empty / non-string rows dropped, packing by characters joined with newlines
    for i in range(2):
        pq.write_table(pa.table({"body": ["aaaa", "", "bbbbbb", None, "cc"][i:]}), str(tmp_path / f"s{i}.parquet"))
    ds = load_response_dataset({"dataset_name": "arrow_text", "data_files": str(tmp_path / "s*.parquet"),
                                "text_key": "body"})
    assert [r["messages"][0]["content"] for r in ds.dataset] == ["aaaa", "bbbbbb", "cc", "bbbbbb", "cc"]
    assert ds.task_name == "x_token" and ds.dataset[0]["messages"][0]["role"] == "assistant"
    ds = load_response_dataset({"dataset_name": "arrow_text", "data_files": str(tmp_path / "s0.parquet"),
                                "text_key": "body", "characters_per_sample": 9})
    assert [r["messages"][0]["content"] for r in ds.dataset] == ["aaaa\nbbbbbb", "cc"]
    tok = get_tokenizer({"name": "byte"})
    d = PROCESSOR_REGISTRY["kd_data_processor"](ds.dataset[1], TaskDataSpec(task_name="x_token"), tok, 256, 0)
    assert d["length"] > 0  # raw-text rows tokenise without a user turn

    # general conversations: role mapping, media aliases, tags consumed in order, media dir lookup
    os.makedirs(tmp_path / "media")
    (tmp_path / "media" / "a.wav").write_bytes(b"RIFF")
    conv = _write_jsonl(tmp_path / "conv.jsonl", [{
        "sound": "a.wav", "image": ["i0.jpg", "i1.jpg"],
        "conversations": [{"from": "human", "value": "Listen <sound> and see <image> <image>"},
                          {"from": "gpt", "value": "ok"}]}])
    ds = load_response_dataset({"dataset_name": "general-conversation-jsonl", "data_path": conv,
                                "media_data_dir": str(tmp_path / "media")})
    user, asst = ds.dataset[0]["messages"]
    assert user["role"] == "user" and asst == {"role": "assistant", "content": [{"type": "text", "text": "ok"}]}
    types = [c["type"] for c in user["content"]]
    assert types == ["text", "audio", "text", "image", "image"]
    assert user["content"][1]["audio"] == str(tmp_path / "media" / "a.wav")  # found under media_data_dir
    assert [c.get("image") for c in user["content"] if c["type"] == "image"] == ["i0.jpg", "i1.jpg"]
    bad = _write_jsonl(tmp_path / "conv_bad.jsonl", [{"conversations": [{"from": "robot", "value": "x"}]}])
    with pytest.raises(ValueError):
        load_response_dataset({"dataset_name": "general-conversation-jsonl", "data_path": bad}).dataset[0]


def test_cascade_sft_and_megatron_packed_sft_rows(tmp_path):
    import warnings

    from rl_b200.data.megatron_sft_packed import IGNORE_INDEX, PROMPT_FORMATS
    from rl_b200.data.response_datasets import load_response_dataset
    from rl_b200.data.tokenizer import get_tokenizer

    casc = _write_jsonl(tmp_path / "casc.jsonl", [{"messages": [{"role": "user", "content": f"q{i}"},
                                                                {"role": "assistant", "content": f"a{i}"}]}
                                                  for i in range(10)])
    ds = load_response_dataset({"dataset_name": "Nemotron-Cascade-2-SFT-Math", "data_path": casc,
                                "max_samples": 4, "split_validation_size": 0.25, "seed": 1})
    assert len(ds.dataset) == 3 and len(ds.val_dataset) == 1 and ds.task_name == "Nemotron-Cascade-2-SFT-Math"

    tok = get_tokenizer({"name": "byte"})
    rec = [{"role": "system", "content": "S"}, {"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"},
           {"role": "system", "content": "T"}, {"role": "user", "content": "q"}, {"role": "assistant", "content": "ok"}]
    path = _write_jsonl(tmp_path / "p.jsonl.packed", [{"conv": rec}])
    cfg = {"dataset_name": "megatron_sft_packed", "data_path": path, "chat_key": "conv",
           "megatron_sft": {"prompt_format": "nemotron-h-aligned"}}
    with pytest.raises(ValueError):  # the policy's CP size is required
        load_response_dataset(cfg)
    ds = load_response_dataset(cfg, context_parallel_size=1)
    row = ds.dataset[0]
    assert row["task_name"] == "megatron_sft_packed" and len(row["packed_messages"]) == 6
    L = 160
    d = ds.processor(row, ds.task_spec, tok, L, 0)
    # expected tokens / labels from the format's rendering, turn by turn
    fmt = PROMPT_FORMATS["nemotron-h-aligned"]
    toks, labs, cu = [], [], [0]
    for conv in (rec[:3], rec[3:]):
        for m in conv:
            ids = tok.encode(fmt.render(m["role"], m["content"]))
            toks += ids
            labs += ids if m["role"] == "assistant" else [IGNORE_INDEX] * len(ids)
        cu.append(len(toks))
    pad = tok.pad_token_id
    cu[-1] = L
    toks += [pad] * (L + 1 - len(toks))
    labs += [pad] * (L + 1 - len(labs))
    assert d["input_ids"].tolist() == toks[:-1] and d["target_ids"].tolist() == labs[1:]
    assert d["packed_cu_seqlens"].tolist() == cu
    exp_mask = [float(t not in (pad, IGNORE_INDEX)) for t in labs[1:]]
    assert d["token_mask"].tolist() == exp_mask and sum(exp_mask) == len(tok.encode("yo\n")) + len(tok.encode("ok\n"))
    pos = d["position_ids"].tolist()
    assert pos[0] == 0 and pos[cu[1]] == 0 and pos[cu[1] - 1] == cu[1] - 1
    # the segment form: (input, target, counted) triples are exactly the pre-shifted row's
    trip = []
    for k, sgm in enumerate(d["packed_segments"]):
        a = cu[k]
        ids, m = sgm["token_ids"].tolist(), sgm["token_loss_mask"].tolist()
        assert len(ids) == cu[k + 1] - a + 1 and m[0] == 0.0
        trip += [(ids[j - 1], ids[j], m[j]) for j in range(1, len(ids))]
    direct = [(d["input_ids"][p].item(), toks[p + 1], d["token_mask"][p].item()) for p in range(L)]
    assert trip == direct

    # context parallelism: every conversation padded to a multiple of 2 * cp; the pack length must be one too
    ds2 = load_response_dataset(cfg, context_parallel_size=2)
    d2 = ds2.processor(row, ds2.task_spec, tok, L, 0)
    seg = (d2["packed_cu_seqlens"][1:] - d2["packed_cu_seqlens"][:-1]).tolist()
    assert all(x % 4 == 0 for x in seg) and d2["packed_context_parallel_size"] == 2
    with pytest.raises(ValueError):
        ds2.processor(row, ds2.task_spec, tok, 90, 0)
    # overflow: the second conversation is cut, with a warning
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        d3 = ds.processor(row, ds.task_spec, tok, cu[1] + 5, 0)
    assert any("overflowed" in str(x.message) for x in w)
    assert d3["packed_cu_seqlens"].tolist() == [0, cu[1], cu[1] + 5] and d3["input_ids"].numel() == cu[1] + 5
    # the identity format trains on every token, the next conversation's first one included
    di = load_response_dataset({**cfg, "megatron_sft": {"prompt_format": "identity"}}, context_parallel_size=1)
    d4 = di.processor(row, di.task_spec, tok, 32, 0)
    n_text = sum(len(m["content"]) for m in rec)
    assert d4["token_mask"].sum().item() == n_text - 1
    with pytest.raises(ValueError):  # unknown option in the megatron_sft block
        load_response_dataset({**cfg, "megatron_sft": {"prompt_format": "identity", "x": 1}}, context_parallel_size=1)


def test_eval_datasets_rekey_and_process(tmp_path):
    import csv

    from rl_b200.data.eval_datasets import load_eval_dataset
    from rl_b200.data.tokenizer import get_tokenizer

    def write_csv(name, header, rows):
        with open(tmp_path / name, "w", newline="") as f:
            w = csv.writer(f)
            w.writerow(header)
            w.writerows(rows)
        return str(tmp_path / name)

    tok = get_tokenizer({"name": "byte"})
    math = write_csv("math_500_test.csv", ["Question", "Answer"], [["1+1?", "2"], ["2*3?", "6"]])
    ds = load_eval_dataset({"dataset_name": "math500", "data_path": math})
    assert ds.task_spec.task_name == "math_500_test" and ds.rekeyed_ds[1] == {"problem": "2*3?", "expected_answer": "6"}
    d = ds.processor(ds.rekeyed_ds[0], ds.task_spec, tok, 256, 0)
    assert d["extra_env_info"]["ground_truth"] == "2" and d["length"] > 0

    mmlu = write_csv("mmlu_DE.csv", ["Question", "A", "B", "C", "D", "Answer", "Subject"],
                     [["q", "a", "b", "c", "d", "C", "physics"]])
    ds = load_eval_dataset({"dataset_name": "mmlu_DE-DE", "data_path": mmlu})
    assert ds.task_spec.task_name == "MMLU_DE-DE" and ds.rekeyed_ds[0]["options"]["C"] == "c"
    d = ds.processor(ds.rekeyed_ds[0], ds.task_spec, tok, 256, 0)
    assert d["extra_env_info"] == {"ground_truth": "C", "subject": "physics"}
    with pytest.raises(ValueError):
        load_eval_dataset({"dataset_name": "mmlu_XX-YY", "data_path": mmlu})

    gp = _write_jsonl(tmp_path / "gpqa.jsonl", [{"Question": f"q{i}", "Correct Answer": "right",
                                                  "Incorrect Answer 1": "w1", "Incorrect Answer 2": "w2",
                                                  "Incorrect Answer 3": "w3"} for i in range(12)])
    a = load_eval_dataset({"dataset_name": "gpqa_diamond", "data_path": gp})
    b = load_eval_dataset({"dataset_name": "gpqa_diamond", "data_path": gp})
    rows = [a.rekeyed_ds[i] for i in range(12)]
    assert rows == [b.rekeyed_ds[i] for i in range(12)]  # seeded: reproducible
    assert all(r["options"][r["answer"]] == "right" for r in rows) and len({r["answer"] for r in rows}) > 1
    assert a.task_spec.task_name == "GPQA_diamond"

    pro = _write_jsonl(tmp_path / "pro.jsonl", [{"question": "q", "options": ["o0", "o1", "o2", "o3", "o4"],
                                                 "answer": "E", "category": "law"}])
    ds = load_eval_dataset({"dataset_name": "mmlu_pro", "data_path": pro})
    assert ds.rekeyed_ds[0]["options"]["E"] == "o4" and ds.task_spec.task_name == "MMLU-Pro"

    local = write_csv("my_set.csv", ["prob", "sol"], [["3+4?", "7"]])
    ds = load_eval_dataset({"dataset_name": local, "problem_key": "prob", "solution_key": "sol", "split": None,
                            "file_format": "csv"})
    assert ds.task_spec.task_name == "my_set" and ds.rekeyed_ds[0]["expected_answer"] == "7"
    with pytest.raises(NotImplementedError):
        load_eval_dataset({"dataset_name": "mmau"})
    # processed for the eval loop: datums with the ground truth for the math environment
    from rl_b200.data.datasets import StatefulDataLoader
    from rl_b200.data.eval_datasets import setup_eval_data

    ds, base = setup_eval_data(tok, {"dataset_name": "math500", "data_path": math, "max_input_seq_length": 128})
    batch = next(iter(StatefulDataLoader(ds, 2, shuffle=False)))
    assert [e["ground_truth"] for e in batch["extra_env_info"]] == ["2", "6"] and batch["length"].min() > 0


def test_setup_response_data_binds_processors_and_envs(tmp_path):
    from rl_b200.data.tokenizer import ByteTokenizer
    from rl_b200.data.utils import setup_response_data
    from rl_b200.environments.math_environment import MathEnvironment

    tr = _write_jsonl(tmp_path / "train.jsonl", _math_rows(12))
    os.makedirs(tmp_path / "val")
    va = _write_jsonl(tmp_path / "val" / "math.jsonl", [{"input": "What is 1 + 1?", "output": "2"}])
    cfg = {"max_input_seq_length": 256,
           "default": {"env_name": "math", "processor": "math_hf_data_processor"},
           "train": {"dataset_name": "OpenMathInstruct-2", "data_path": tr, "split_validation_size": 0.25},
           "validation": [{"dataset_name": "ResponseDataset", "data_path": va}]}
    tok = ByteTokenizer()
    train, val, t2e, v2e = setup_response_data(tok, cfg, {"math": {}})
    assert len(train) == 9 and len(val) == 3 + 1
    assert isinstance(t2e["OpenMathInstruct-2"], MathEnvironment) and set(v2e) == {"OpenMathInstruct-2", "val-math"}
    d = train[0]
    assert d["task_name"] == "OpenMathInstruct-2" and d["extra_env_info"]["ground_truth"].isdigit()
    assert val[3]["extra_env_info"] == {"ground_truth": "2"}
    # the environment verifies the decoded response against the ground truth
    env = t2e["OpenMathInstruct-2"]
    resp = torch.tensor(tok.encode("so the answer is \\boxed{2}"))
    ret = env.step([[{"role": "assistant", "token_ids": resp}]], [{"ground_truth": "2"}])
    assert float(ret.rewards[0]) == 1.0


def test_grpo_trains_on_jsonl_math_set_through_run_grpo(tmp_path):
    from examples.run_grpo import main

    tr = _write_jsonl(tmp_path / "math.jsonl", _math_rows(32))
    state = main(["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  "logger.log_dir=" + str(tmp_path / "logs"), "logger.stdout=false",
                  "policy.max_total_sequence_length=96", "policy.generation.max_new_tokens=16",
                  "+policy.tokenizer.name=byte",
                  "~data.num_prompts", "~data.min_prompt_len", "~data.max_prompt_len",
                  "+data.max_input_seq_length=80",
                  "+data.train.dataset_name=ResponseDataset", f"+data.train.data_path={tr}",
                  "+data.train.input_key=problem", "+data.train.output_key=expected_answer",
                  "+data.train.env_name=math", "~env.synthetic", "+env.math.kind=math"])
    assert state["current_step"] == 2
