"""Chat client helpers, the project-size snapshot and multimodal collation."""

import json

import pytest
import torch

from wavelet_b200.data.multimodal import collate_multimodal_fields
from wavelet_b200.tools import chat, project_size


def test_reply_text():
    assert chat.reply_text({"choices": [{"message": {"content": "hi"}}]}) == "hi"
    tc = [{"id": "1", "function": {"name": "f", "arguments": "{}"}}]
    assert json.loads(chat.reply_text({"choices": [{"message": {"content": None, "tool_calls": tc}}]})) == tc
    with pytest.raises(RuntimeError):
        chat.reply_text({"choices": []})


def test_project_size(tmp_path):
    (tmp_path / "wavelet_b200" / "ops").mkdir(parents=True)
    (tmp_path / "wavelet_b200" / "ops" / "a.py").write_text("# c\n\ndef f(x):\n    if x:\n        return 1\n")
    (tmp_path / "tests").mkdir()
    (tmp_path / "tests" / "t.cu").write_text("// k\n__global__ void k() {}\n")
    files = [project_size.measure(tmp_path, p) for p in project_size.project_files(tmp_path)]
    snap = project_size.summarize(files, timestamp="t")
    assert snap["files"] == 2 and snap["python_functions"] == 1 and snap["python_complexity_points"] == 1
    assert snap["by_category"]["ops"]["source_lines"] == 3 and snap["by_category"]["tests"]["source_lines"] == 1


def test_multimodal_collation():
    s = [{"input_ids": [1, 2, 3], "mm_kwargs": {"pixel_values": torch.ones(4, 8), "mm_token_type_ids": [0, 1, 1]}},
         {"input_ids": [1, 2], "mm_kwargs": {"pixel_values": torch.zeros(2, 8), "mm_token_type_ids": [1, 0]}}]
    out = collate_multimodal_fields(s, max_len=5)
    assert out["pixel_values"].shape == (6, 8)
    assert out["mm_token_type_ids"].tolist() == [[0, 1, 1, 0, 0], [1, 0, 0, 0, 0]]
    with pytest.raises(ValueError):
        collate_multimodal_fields([{"input_ids": [1], "mm_kwargs": {"audio": [1]}}], 2)
    with pytest.raises(ValueError):
        collate_multimodal_fields([s[0], {"input_ids": [1], "mm_kwargs": {}}], 4)
