"""Disaggregated prefill / decode: moving a request's KV cache from a prefill engine to a
decode engine.  See :mod:`.connector`."""
from .connector import KVTransferConfig, TorchDistKVConnector

__all__ = ["KVTransferConfig", "TorchDistKVConnector"]
