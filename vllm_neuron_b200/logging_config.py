"""Logger set-up (parity with ``vllm_neuron/logging_config.py:14``)."""

from __future__ import annotations

import logging
import sys

_CONFIGURED = False


def setup_logging() -> logging.Logger:
    global _CONFIGURED
    from . import envs

    logger = logging.getLogger("vllm_neuron_b200")
    if not _CONFIGURED:
        handler = logging.StreamHandler(sys.stderr)
        handler.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s:%(lineno)d] %(message)s"))
        logger.addHandler(handler)
        logger.propagate = False
        _CONFIGURED = True
    logger.setLevel(getattr(logging, str(envs.VLLM_B200_LOG_LEVEL).upper(), logging.INFO))
    return logger


def init_logger(name: str) -> logging.Logger:
    setup_logging()
    return logging.getLogger(name if name.startswith("vllm_neuron_b200") else f"vllm_neuron_b200.{name}")
