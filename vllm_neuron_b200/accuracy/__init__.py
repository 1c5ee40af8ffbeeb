"""Accuracy tooling: logit validation against a reference model, three-way closeness checks and
hidden-state capture (reference: vllm_neuron/accuracy/logit_validation.py, tensor_capture.py,
testing.py ``assert_close_three_way``)."""
from .logit_validation import LogitReport, assert_close_three_way, capture_hidden, compare_logits, validate_against_hf

__all__ = ["LogitReport", "assert_close_three_way", "capture_hidden", "compare_logits", "validate_against_hf"]
