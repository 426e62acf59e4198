"""Errors of the operator surface, mirroring crates/runtimed-model/src/error.rs:6-27 (ModelError)."""
from __future__ import annotations


class ModelError(Exception):
    """Base of every error the operator surface raises."""


class ConfigError(ModelError):
    """ModelError::Config -- a bad configuration or a failed device call."""


class MissingWeight(ModelError, KeyError):
    """ModelError::MissingWeight(name)."""

    def __init__(self, name: str):
        super().__init__(f"missing weight: {name}")
        self.name = name

    def __str__(self) -> str:  # KeyError would quote the message
        return f"missing weight: {self.name}"


class ShapeError(ModelError):
    """ModelError::Shape { name, expected, got }."""

    def __init__(self, name: str, expected, got):
        super().__init__(f"shape mismatch on {name}: expected {list(expected)}, got {list(got)}")
        self.name = name
        self.expected = list(expected)
        self.got = list(got)


class GgufError(ModelError):
    """ModelError::Gguf -- Unsupported / Truncated / Overflow from the GGUF layer."""
