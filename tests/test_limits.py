"""Output-length clamping; the reference's own cases (tests/test_limits.py:9-21)."""

from gemma4_b200.limits import DEFAULT_CONTEXT_TOKENS, MAX_OUTPUT_TOKENS, allowed_output_tokens


def test_request_below_limit_is_unchanged():
    assert allowed_output_tokens(5000, 54, 32768) == 5000


def test_model_limit_is_reduced_to_fit_prompt():
    assert allowed_output_tokens(32768, 54, 32768) == 32714


def test_oversized_request_is_clamped():
    assert allowed_output_tokens(128000, 54, 32768) == 32714


def test_full_prompt_has_no_output_capacity():
    assert allowed_output_tokens(5000, 32768, 32768) == 0


def test_minimum_one_token_and_constants():
    assert allowed_output_tokens(0, 10, 100) == 1
    assert MAX_OUTPUT_TOKENS == DEFAULT_CONTEXT_TOKENS == 32768
