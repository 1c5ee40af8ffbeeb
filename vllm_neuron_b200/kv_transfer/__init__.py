"""Disaggregated serving: moving a request's KV cache from a prefill engine to a decode engine,
and vision-encoder outputs from an encoder instance to a prefill/decode instance.  See
:mod:`.connector`."""
from .connector import ECTransferConfig, KVTransferConfig, TensorChannel, TorchDistKVConnector

__all__ = ["ECTransferConfig", "KVTransferConfig", "TensorChannel", "TorchDistKVConnector"]
