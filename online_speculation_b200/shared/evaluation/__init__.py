"""Benchmark loading and deterministic answer evaluation."""

from .consensus import CumulativeConsensusReward, consensus_index, modal_answer
from .gsm8k import (GSM8K_PROMPT_SUFFIX, GSM8K_TEST_SHA256, GSM8K_TEST_URL, GSM8K_TRAIN_SHA256, GSM8K_TRAIN_URL,
                    GSM8KProblem, accuracy, download_gsm8k, gsm8k_prompt, load_gsm8k, select_problems)
from .numeric import NumericReferenceVerifier, build_numeric_reference_verifier, extract_numeric_answer

__all__ = ["CumulativeConsensusReward", "GSM8KProblem", "GSM8K_PROMPT_SUFFIX", "GSM8K_TEST_SHA256", "GSM8K_TEST_URL",
           "GSM8K_TRAIN_SHA256", "GSM8K_TRAIN_URL", "NumericReferenceVerifier", "accuracy",
           "build_numeric_reference_verifier", "consensus_index", "download_gsm8k", "extract_numeric_answer",
           "gsm8k_prompt", "load_gsm8k", "modal_answer", "select_problems"]
