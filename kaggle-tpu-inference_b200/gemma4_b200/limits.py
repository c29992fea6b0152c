"""Context limits of the resident-cache configuration (reference gemma4_tpu/limits.py:1-8)."""

MAX_OUTPUT_TOKENS = 32768
DEFAULT_CONTEXT_TOKENS = 32768


def allowed_output_tokens(requested: int, prompt_tokens: int, context_tokens: int) -> int:
    """Clamp a request to [1, MAX_OUTPUT_TOKENS] and to the context left after the prompt."""
    room = context_tokens - prompt_tokens
    if room <= 0:
        return 0
    return min(max(1, requested), MAX_OUTPUT_TOKENS, room)
