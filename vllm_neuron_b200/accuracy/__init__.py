"""Accuracy tooling: logit validation against a reference model, three-way closeness checks,
hidden-state capture, activation capture / golden replacement keyed by request and position, and
capture comparison with divergence localisation, and KV-cache analysis (reference:
vllm_neuron/accuracy/logit_validation.py, tensor_capture.py, tensor_replacement.py,
tensor_compare.py, kv_cache_analysis.py, testing.py ``assert_close_three_way``)."""
from .logit_validation import LogitReport, assert_close_three_way, capture_hidden, compare_logits, validate_against_hf
from .tensor_capture import CaptureSession, TensorCapture, TensorReplacement, expand_patterns, session_from_config
from .kv_cache_analysis import (KVComparison, KVSet, compare_kv_caches, extract_request_kv, format_kv_report,
                                hf_kv)
from .tensor_compare import compare_captures, compare_tensors, first_divergence, format_report

__all__ = ["LogitReport", "assert_close_three_way", "capture_hidden", "compare_logits", "validate_against_hf",
           "CaptureSession", "TensorCapture", "TensorReplacement", "expand_patterns", "session_from_config",
           "compare_captures", "compare_tensors", "first_divergence", "format_report",
           "KVComparison", "KVSet", "compare_kv_caches", "extract_request_kv", "format_kv_report", "hf_kv"]
