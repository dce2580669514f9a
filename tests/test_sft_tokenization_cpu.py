"""SFT loss masks against the reference's tokenization tests
(tests/test_tokenization_alignment.py of the reference): only completion
content is trained (role headers and context are not), ``step_loss_mask: 0``
switches a turn off, ``data.loss_mask.tool`` trains tool turns, truncation
keeps the trainable prefix."""

from types import SimpleNamespace

from wavelet_b200.configs.config import LossMaskConfig
from wavelet_b200.data.sft import tokenize_messages
from wavelet_b200.data.tokenizer import CharTokenizer

TOK = CharTokenizer()


def _trained(msgs, **lm):
    s = tokenize_messages(msgs, TOK, SimpleNamespace(loss_mask=LossMaskConfig(**lm)))
    ids = [t for t, m in zip(s.input_ids, s.loss_mask) if m]
    return TOK.decode(ids), ids


def test_only_assistant_completion_is_trained():
    text, ids = _trained([{"role": "system", "content": "rules"}, {"role": "user", "content": "hi"},
                          {"role": "assistant", "content": "ok"}])
    assert text == "ok\n" and ids[-1] == TOK.eos_token_id


def test_step_loss_mask_switches_a_turn_off():
    text, _ = _trained([{"role": "user", "content": "run"},
                        {"role": "assistant", "content": "tool call", "step_loss_mask": 0},
                        {"role": "tool", "content": "result"}, {"role": "assistant", "content": "done"}])
    assert text == "done\n"


def test_tool_turns_train_when_configured():
    text, _ = _trained([{"role": "user", "content": "lookup"},
                        {"role": "assistant", "content": "call", "step_loss_mask": 0},
                        {"role": "tool", "content": "42"}, {"role": "assistant", "content": "answer"}], tool=True)
    assert "42" in text and text.endswith("answer\n") and "call" not in text


def test_hf_style_template_masks_the_generation_prompt():
    class Templated:  # a chat template with a distinct generation prompt and end token
        eos_token_id = 0

        def apply_chat_template(self, msgs, tokenize=True, add_generation_prompt=False):
            out = []
            for m in msgs:
                out += [100 + ["system", "user", "assistant", "tool"].index(m["role"])] + [ord(c) for c in m["content"]] + [9]
            return out + ([102] if add_generation_prompt else [])

    s = tokenize_messages([{"role": "user", "content": "hi"}, {"role": "assistant", "content": "ok"}], Templated(),
                          SimpleNamespace(loss_mask=LossMaskConfig()))
    assert [t for t, m in zip(s.input_ids, s.loss_mask) if m] == [ord("o"), ord("k"), 9]


def test_cat_packing_resume_keeps_the_pending_sample():
    from wavelet_b200.configs.config import SFTConfig
    from wavelet_b200.data.sft import SFTDataset

    cfg = SFTConfig.model_validate({"data": {"source": "fake", "seq_len": 64, "micro_batch_size": 1,
                                             "pack_function": "cat", "fake_length": "variable",
                                             "max_examples": 12, "batch_size": 1}}).data
    a = SFTDataset(cfg, seed=3)
    for _ in range(3):
        a.next_micro_batch()
    sd = a.state_dict()
    b = SFTDataset(cfg, seed=3)
    b.load_state_dict(sd)
    for _ in range(4):
        x, y = a.next_micro_batch(), b.next_micro_batch()
        assert x.input_ids.tolist() == y.input_ids.tolist()
