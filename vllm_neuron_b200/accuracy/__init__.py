"""Accuracy tooling: logit validation against a reference model, three-way closeness checks,
hidden-state capture, activation capture / golden replacement keyed by request and position, and
capture comparison with divergence localisation (reference: vllm_neuron/accuracy/
logit_validation.py, tensor_capture.py, tensor_replacement.py, tensor_compare.py, testing.py
``assert_close_three_way``)."""
from .logit_validation import LogitReport, assert_close_three_way, capture_hidden, compare_logits, validate_against_hf
from .tensor_capture import CaptureSession, TensorCapture, TensorReplacement, expand_patterns, session_from_config
from .tensor_compare import compare_captures, compare_tensors, first_divergence, format_report

__all__ = ["LogitReport", "assert_close_three_way", "capture_hidden", "compare_logits", "validate_against_hf",
           "CaptureSession", "TensorCapture", "TensorReplacement", "expand_patterns", "session_from_config",
           "compare_captures", "compare_tensors", "first_divergence", "format_report"]
