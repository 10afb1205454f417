"""Attribution: attributors, their configuration and the score container."""

from dattri_llm_b200.attribution.algorithm import TracInAttributor
from dattri_llm_b200.attribution.arguments import AttributionArguments
from dattri_llm_b200.attribution.base import BaseAttributor, BaseInnerProductAttributor
from dattri_llm_b200.attribution.score import AttributionScore

__all__ = ["AttributionArguments", "AttributionScore", "BaseAttributor", "BaseInnerProductAttributor",
           "TracInAttributor"]
