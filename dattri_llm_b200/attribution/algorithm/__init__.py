"""Attribution algorithms."""

from dattri_llm_b200.attribution.algorithm.adamw_influence import AdamWInfluenceAttributor
from dattri_llm_b200.attribution.algorithm.dvemb import DVEmbAttributor
from dattri_llm_b200.attribution.algorithm.kronecker import EKFACAttributor, KFACAttributor, KroneckerAttributor
from dattri_llm_b200.attribution.algorithm.less import LESSAttributor
from dattri_llm_b200.attribution.algorithm.tracin import TracInAttributor
from dattri_llm_b200.attribution.algorithm.trajectory import TrajectoryAttributor

__all__ = ["AdamWInfluenceAttributor", "DVEmbAttributor", "EKFACAttributor", "KFACAttributor",
           "KroneckerAttributor", "LESSAttributor", "TracInAttributor", "TrajectoryAttributor"]
