"""Host logic of nekochat_b200.generate (the engine's prefix reuse and prefill chunking, engine.cpp:74-112)."""
from nekochat_b200.generate import common_prefix, fit_prompt, prefill_chunks


def test_common_prefix_keeps_one_token_to_rerun():
    assert common_prefix([], [5, 6, 7]) == 0
    assert common_prefix([5, 6, 9], [5, 6, 7]) == 2
    assert common_prefix([5, 6, 7], [5, 6, 7]) == 2        # identical prompt: the last token is re-run
    assert common_prefix([5, 6, 7, 8], [5, 6]) == 1        # shorter prompt inside the cache
    assert common_prefix([5], [5, 6, 7]) == 1
    assert common_prefix([1], [2]) == 0


def test_fit_prompt_empty_and_overlong():
    assert fit_prompt([], 16, eos=3) == [3]
    assert fit_prompt(list(range(20)), 16) == list(range(5, 20))   # context - 1 last tokens
    assert fit_prompt(list(range(15)), 16) == list(range(15))


def test_prefill_chunks_end_before_the_last_token():
    assert prefill_chunks(0, 10, 64) == [(0, 9), (9, 10)]
    assert prefill_chunks(0, 130, 64) == [(0, 64), (64, 128), (128, 129), (129, 130)]
    assert prefill_chunks(0, 65, 64) == [(0, 64), (64, 65)]
    assert prefill_chunks(7, 8, 64) == [(7, 8)]
    assert prefill_chunks(0, 1, 64) == [(0, 1)]
