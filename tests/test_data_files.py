"""File datasets (parquet / jsonl in the reference row layout): prompt
rendering, metadata for the reward loops, overlong filtering, seeded
per-epoch order, resume cursor, validation rows and a training run."""

import json

import pyarrow as pa
import pyarrow.parquet as pq

from psrl_b200.agent.data import DataProcessor
from psrl_b200.config import load_config


def _rows(n=6):
    return [{"prompt": [{"role": "user", "content": f"What is {i} + {i}?"}], "data_source": "gsm8k",
             "reward_model": {"ground_truth": str(2 * i)}, "extra_info": {"index": i}} for i in range(n)]


def _cfg(tmp_path, fmt="parquet", rows=None, *extra):
    rows = rows or _rows()
    if fmt == "parquet":
        path = str(tmp_path / "train.parquet")
        pq.write_table(pa.Table.from_pylist(rows), path)
    else:
        path = str(tmp_path / "train.jsonl")
        with open(path, "w") as fh:
            fh.writelines(json.dumps(r) + "\n" for r in rows)
    return load_config(preset="cpu_tiny_grpo", overrides=[f"data.kind={fmt}", f"data.train_files={path}", *extra])


def test_parquet_rows_become_prompt_groups(tmp_path):
    cfg = _cfg(tmp_path)
    dp = DataProcessor(cfg, 1024, 4)
    items = [dp.next_group() for _ in range(6)]
    texts = {dp.tokenizer.decode(it.prompt_ids) for it in items}
    assert len(texts) == 6 and all("<|im_start|>assistant" in t for t in texts)
    it = items[0]
    i = int(it.meta["extra_info"]["index"])
    assert it.meta["data_source"] == "gsm8k" and it.meta["ground_truth"] == str(2 * i)
    assert f"What is {i} + {i}?" in dp.tokenizer.decode(it.prompt_ids)
    # next epoch: a different seeded order of the same rows; a restarted processor replays it
    ep2 = [dp.tokenizer.decode(dp.next_group().prompt_ids) for _ in range(6)]
    assert set(ep2) == texts
    dp2 = DataProcessor(cfg, 1024, 4)
    dp2.load_state_dict({"cursor": 6})
    assert [dp2.tokenizer.decode(dp2.next_group().prompt_ids) for _ in range(6)] == ep2


def test_jsonl_overlong_filter_and_string_prompts(tmp_path):
    rows = _rows(3) + [{"prompt": "x" * 500, "answer": 1}, {"prompt": "short one", "answer": 7}]
    cfg = _cfg(tmp_path, "jsonl", rows)
    dp = DataProcessor(cfg, 1024, 2)
    assert dp.src.dropped == 1 and len(dp.src.items) == 4
    metas = [dp.src.item(k).meta for k in range(4)]
    assert any(m["ground_truth"] == 7 for m in metas)
    val = dp.validation_items(2)
    assert [v.prompt_ids for v in val] == [dp.src.items[0][0], dp.src.items[1][0]]


def test_training_on_a_parquet_dataset(tmp_path):
    import torch
    torch.set_num_threads(2)
    from psrl_b200.trainer import RLTrainer
    cfg = _cfg(tmp_path, "parquet", _rows(12), "reward.kind=naive", "++reward.task=addition",
               "rollout.max_response_length=8")
    t = RLTrainer(cfg)
    out = t.fit(1)
    t.stop_rollout()
    assert out[0]["num_trajectories"] == 32


def test_unshuffled_file_order(tmp_path):
    cfg = _cfg(tmp_path, "jsonl", None, "data.shuffle=false")
    dp = DataProcessor(cfg, 1024, 2)
    got = [dp.next_group().meta["extra_info"]["index"] for _ in range(8)]
    assert got == [0, 1, 2, 3, 4, 5, 0, 1]
