"""Accuracy toolkit: tolerance checks (two- and three-way), logit validation against a
reference model, tensor capture / replacement hooks and KV-cache inspection."""

from .logit_validation import (compare_logits, logit_validation, make_engine_generate_fn,  # noqa: F401
                               multi_prompt_logit_validation, validate_greedy_generation, validate_prompt_logits)
from .testing import assert_close, assert_close_three_way, compare  # noqa: F401
