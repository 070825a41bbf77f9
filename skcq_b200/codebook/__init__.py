"""B200 drop-in for ``skcq.codebook``: the same public names and contracts."""

from __future__ import annotations

from skcq_b200.codebook.aqlm import AQLMCodebook, AQLMCodebookConfig
from skcq_b200.codebook.base import DistanceMetric, WeightsCodebookBase
from skcq_b200.codebook.cwr import AQLMCWR, SSVQCWR, CompressedWeightsRepresentation, EuclideanCWR, SphericalCWR
from skcq_b200.codebook.euclidean import EuclideanCodebook, EuclideanCodebookConfig
from skcq_b200.codebook.events import (
    CodebookDoneEvent,
    CodebookIterEvent,
    CodebookStartEvent,
    Experiment,
    KmeansDoneEvent,
    KmeansIterEvent,
    KmeansStartEvent,
    TqdmListener,
)
from skcq_b200.codebook.kmeans import KmeansConfig, KmeansExperiment
from skcq_b200.codebook.spherical import (
    ScaleQuantState,
    SphericalCodebook,
    SphericalCodebookConfig,
    parse_scale_dtype,
    quantize_spherical_scales,
    scale_bits_per_elem,
)
from skcq_b200.codebook.ssvq import SSVQCodebook

__all__ = [
    "WeightsCodebookBase", "DistanceMetric",
    "CompressedWeightsRepresentation", "EuclideanCWR", "SphericalCWR", "SSVQCWR", "AQLMCWR",
    "EuclideanCodebook", "EuclideanCodebookConfig", "SphericalCodebook", "SphericalCodebookConfig",
    "SSVQCodebook", "AQLMCodebook", "AQLMCodebookConfig",
    "ScaleQuantState", "quantize_spherical_scales", "scale_bits_per_elem", "parse_scale_dtype",
    "Experiment", "KmeansStartEvent", "KmeansIterEvent", "KmeansDoneEvent",
    "CodebookStartEvent", "CodebookIterEvent", "CodebookDoneEvent", "TqdmListener",
    "KmeansConfig", "KmeansExperiment",
]
