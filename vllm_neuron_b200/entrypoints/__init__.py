from .llm import LLM

__all__ = ["LLM"]
