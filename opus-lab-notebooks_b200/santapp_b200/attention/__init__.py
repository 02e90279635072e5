"""SANTA++ attention: cluster summary, sparse decode, mini-batch k-means."""

from .santapp import (ClusterSummary, DecodeResult, DecodeTrafficTracker,  # noqa: F401
                      DecodeStep, DecodeWorkspace, GraphedDecodeStep, allocate_summary,
                      build_summary, santa_decode, santa_decode_select)
from .paged import PagedKVCache  # noqa: F401
