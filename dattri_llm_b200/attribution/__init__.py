"""Attribution: attributors, their configuration and the score container."""

from dattri_llm_b200.attribution.algorithm import (
    AdamWInfluenceAttributor,
    DVEmbAttributor,
    EKFACAttributor,
    KFACAttributor,
    KroneckerAttributor,
    LESSAttributor,
    TracInAttributor,
    TrajectoryAttributor,
)
from dattri_llm_b200.attribution.arguments import AttributionArguments
from dattri_llm_b200.attribution.base import BaseAttributor, BaseInnerProductAttributor
from dattri_llm_b200.attribution.score import AttributionScore

__all__ = ["AdamWInfluenceAttributor", "AttributionArguments", "AttributionScore", "BaseAttributor",
           "BaseInnerProductAttributor", "DVEmbAttributor", "EKFACAttributor", "KFACAttributor",
           "KroneckerAttributor", "LESSAttributor", "TracInAttributor", "TrajectoryAttributor"]
