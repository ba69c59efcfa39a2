"""CPU checks of the `GreedyDecodeEngine` drop-in's request rules
(greedy_engine.py; the reference's evaluation_wrapper.py:98-127 plus this
engine's cache bound).  No engine is built: the checks need no GPU."""
import torch

from greedy_engine import GreedyDecodeEngine


class _Eng:
    max_cache_len = 64


def _engine(threshold=16):
    g = object.__new__(GreedyDecodeEngine)
    g._max_tokens_threshold = threshold
    g._engine = _Eng()
    return g


def test_request_rules_follow_the_reference():
    g = _engine()
    ids = torch.zeros((1, 10), dtype=torch.long)
    assert g.is_supported((ids,), {"max_new_tokens": 8})
    assert g.is_supported((), {"input_ids": ids, "attention_mask": torch.ones(1, 10), "max_new_tokens": 16})
    reason = g._get_support_failure_reason
    assert "len(args)" in reason((ids, ids), {})
    assert "unsupported kwargs" in reason((ids,), {"top_k": 5})
    assert "rank-2" in reason((ids[0],), {})
    assert "batch_size" in reason((torch.zeros((2, 10), dtype=torch.long),), {})
    assert "do_sample" in reason((ids,), {"do_sample": True})
    assert "use_cache" in reason((ids,), {"use_cache": False})
    assert "max_new_tokens must be" in reason((ids,), {"max_new_tokens": 0})
    assert "exceeds threshold" in reason((ids,), {"max_new_tokens": 17})
    assert "padding" in reason((ids,), {"attention_mask": torch.tensor([[0] + [1] * 9])})
    assert "exceeds the cache" in reason((torch.zeros((1, 60), dtype=torch.long),), {"max_new_tokens": 8})
    assert reason((torch.zeros((1, 57), dtype=torch.long),), {"max_new_tokens": 8}) is None


def test_eos_resolution_order():
    class Cfg:
        def get_text_config(self, decoder=True):
            return type("T", (), {"eos_token_id": 7})()

    class Model:
        config = Cfg()
        generation_config = type("G", (), {"eos_token_id": [5, 6]})()

    g = _engine()
    g._model = Model()
    assert g._eos_values({"eos_token_id": 3}) == [3]
    assert g._eos_values({"eos_token_id": torch.tensor([3, 4])}) == [3, 4]
    assert g._eos_values({}) == [5, 6]
    Model.generation_config = None
    assert g._eos_values({}) == [7]
