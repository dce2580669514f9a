"""Multi-turn token merging against the cases the reference's trajectory
tests pin (tests/test_agent_trajectory.py of the reference).  Rows here are
aligned to ``input_ids`` (the output token itself is marked), where the
reference lists shifted targets; the trained tokens, log-probs and masks are
the same."""

import itertools
import random

import pytest

from wavelet_b200.data.rl import sample_from_example
from wavelet_b200.orchestrator.agent_trajectory import (TokenSegment, _unique_ordered_output_matches,
                                                        merge_token_segments, to_rl_example)


def _trained(row, field):
    return [v for v, m in zip(getattr(row, field), row.loss_mask) if m]


def test_unique_ordered_matches_agree_with_exhaustive_search():
    rng = random.Random(31)
    cases = [([[1], [2]], [2, 1, 2, 1]), ([[1, 1], [1, 1]], [1] * 4), ([[1, 1], [1, 1]], [1] * 5),
             ([[1, 2], [1]], [1, 2]), ([[]], [1]), ([], [])]
    cases += [([[rng.randrange(2) for _ in range(rng.randrange(1, 5))] for _ in range(rng.randrange(1, 4))],
               [rng.randrange(2) for _ in range(rng.randrange(13))]) for _ in range(500)]
    for outs, prompt in cases:
        places = itertools.product(*[[i for i in range(len(prompt) - len(o) + 1) if o and prompt[i:i + len(o)] == o]
                                     for o in outs])
        valid = [list(p) for p in places if all(p[i] + len(outs[i]) <= p[i + 1] for i in range(len(p) - 1))]
        assert _unique_ordered_output_matches(outs, prompt) == (valid[0] if len(valid) == 1 else None), (outs, prompt)
    long = list(range(1024))
    assert _unique_ordered_output_matches([[t] for t in long], long) == long


def test_exact_prefix_merges_turns():
    (row,) = merge_token_segments([TokenSegment([1, 2], [3, 4], [-0.3, -0.4], turn_id="turn-0"),
                                   TokenSegment([1, 2, 3, 4, 5], [6], [-0.6], turn_id="turn-1")], temperature=0.7)
    assert row.input_ids == [1, 2, 3, 4, 5, 6]
    assert row.loss_mask == [False, False, True, True, False, True]
    assert _trained(row, "inference_logprobs") == [-0.3, -0.4, -0.6]
    assert row.temperatures == [0.7] * 6
    assert row.turn_ids == ["turn-0"] * 4 + ["turn-1"] * 2


def test_non_extending_prompt_fans_out_and_ambiguity_is_rejected():
    rows = merge_token_segments([TokenSegment([1, 2], [3], [-0.3]), TokenSegment([1, 9], [10], [-0.1])])
    assert [r.input_ids for r in rows] == [[1, 2, 3], [1, 9, 10]]
    rows = merge_token_segments([TokenSegment([1, 2], [3, 4], [-0.3, -0.4]),
                                 TokenSegment([1, 3, 4, 5, 3, 4], [6], [-0.6])])
    assert [r.input_ids for r in rows] == [[1, 2, 3, 4], [1, 3, 4, 5, 3, 4, 6]]


def test_rerendered_history_is_rebased():
    segs = [TokenSegment([1, 10, 11, 20, 21, 22], [30, 31], [-0.3, -0.31], output_sampling_mask=[[30, 130], [31, 131]],
                         turn_id="turn-0"),
            TokenSegment([1, 10, 11, 20, 30, 31, 40, 20, 21, 22], [50, 51], [-0.5, -0.51],
                         output_sampling_mask=[[50, 150], [51, 151]], turn_id="turn-1"),
            TokenSegment([1, 10, 11, 20, 30, 31, 40, 20, 50, 51, 60, 20, 21, 22], [70], [-0.7],
                         output_sampling_mask=[[70, 170]], turn_id="turn-2")]
    (row,) = merge_token_segments(segs, temperature=0.8)
    assert _trained(row, "input_ids") == [30, 31, 50, 51, 70]
    assert _trained(row, "inference_logprobs") == [-0.3, -0.31, -0.5, -0.51, -0.7]
    assert _trained(row, "sampling_masks") == [[30, 130], [31, 131], [50, 150], [51, 151], [70, 170]]
    assert row.input_ids == [1, 10, 11, 20, 30, 31, 40, 20, 50, 51, 60, 20, 21, 22, 70]
    ex = to_rl_example(row, reward=1.0, advantage=0.5)
    s = sample_from_example(ex)  # the trainer's alignment accepts the row
    assert s.loss_mask.sum().item() == 5
    assert [m for m in s.sampling_mask if m] == [[30, 130], [31, 131], [50, 150], [51, 151], [70, 170]]


def test_masked_outputs_keep_logprobs_and_media_changes_split():
    (row,) = merge_token_segments([TokenSegment([1], [2, 3], [-0.2, -0.3])], mask_outputs=True)
    assert row.loss_mask == [False, False, False] and row.inference_logprobs == [0.0, -0.2, -0.3]
    with pytest.raises(ValueError, match="output_logprobs"):
        TokenSegment([1], [2, 3], [-0.2])
    rows = merge_token_segments([TokenSegment([1, 2], [3], [-1.0], metadata={"media_fingerprint": "red"}),
                                 TokenSegment([1, 2, 3, 4], [5], [-2.0], metadata={"media_fingerprint": "blue"})])
    assert [r.terminal_segment_index for r in rows] == [0, 1]
    assert [sum(r.loss_mask) for r in rows] == [1, 1]
