"""Attribution algorithms."""

from dattri_llm_b200.attribution.algorithm.tracin import TracInAttributor

__all__ = ["TracInAttributor"]
