"""Torch-CPU restatement of the reference's per-head SANTA++ decode, for the
hybrid estimator ("top-k clusters plus N sampled tokens").

TEST AND BASELINE INFRASTRUCTURE ONLY.  ``bench.py`` times it as the CPU
baseline and as the reference arm (the reference's own code is Python over
torch and does not travel to the GPU machines); ``tests/`` check it against
the oracle (``santa_oracle.decode_hybrid``).  The product package never
imports it.

It follows the op structure of the reference's ``SantaPlusEngine``
(santapp-ruler-bench/src/santapp_ruler/attention/santapp.py), one call per
(sequence, query head) on the host, with torch's intra-op threads:

* ``build_summary``: santapp.py:508-540 (bincount, drop empty clusters,
  members by a stable argsort of the labels, exclusive cumsum starts,
  ``index_add_`` centroid sums divided by the counts);
* ``approximate_attention_hybrid``: the recent window of santapp.py:379-388;
  the guess ``log n + C q scale`` and descending argsort of santapp.py:397-401
  cut at k clusters, their members gathered as in 402-411; uniform samples
  over the remaining old-prefix tokens with ``log r = -log(n_rest)``
  (santapp.py:459-468, restricted to the non-selected tokens); the
  self-normalised combine and ESS of santapp.py:472-506 with the selected
  clusters' tokens as exact terms.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class TorchSummary:
    members: torch.Tensor        # int64 [N] token ids sorted by cluster
    starts: torch.Tensor         # int64 [G'] start of each non-empty cluster
    lengths_long: torch.Tensor   # int64 [G']
    lengths_float: torch.Tensor  # fp32 [G']
    key_centroids: torch.Tensor  # fp32 [G', D]

    @property
    def num_groups(self) -> int:
        return int(self.lengths_long.numel())


def build_summary(keys: torch.Tensor, labels: torch.Tensor, n_clusters: int) -> TorchSummary:
    """santapp.py:508-540 on the old-prefix keys [N, D] (fp32 upcast)."""
    keys = keys.float()
    labels = labels.long()
    counts = torch.bincount(labels, minlength=n_clusters)
    nonempty = counts > 0
    members = torch.argsort(labels, stable=True)
    starts_all = torch.zeros(n_clusters, dtype=torch.long)
    starts_all[1:] = torch.cumsum(counts, 0)[:-1]
    sums = torch.zeros(n_clusters, keys.shape[1], dtype=torch.float32)
    sums.index_add_(0, labels, keys)
    n = counts[nonempty]
    return TorchSummary(members=members, starts=starts_all[nonempty].contiguous(),
                        lengths_long=n.contiguous(), lengths_float=n.float(),
                        key_centroids=(sums[nonempty] / n[:, None].float()).contiguous())


def rest_positions(summary: TorchSummary, chosen: torch.Tensor,
                   ranks: torch.Tensor) -> torch.Tensor:
    """Member positions of ranks in [0, n_rest): the r-th position outside
    the chosen clusters, positions in ascending order."""
    st = summary.starts[chosen]
    ln = summary.lengths_long[chosen]
    order = torch.argsort(st)
    st, ln = st[order], ln[order]
    before = torch.cumsum(ln, 0) - ln              # chosen positions before cluster j
    gap = st - before                               # non-chosen positions before cluster j
    j = torch.searchsorted(gap, ranks, right=True)  # clusters wholly before the rank
    cum = torch.cat((torch.zeros(1, dtype=torch.long), torch.cumsum(ln, 0)))
    return ranks + cum[j]


@dataclass
class HeadResult:
    out: torch.Tensor   # fp32 [D]
    ess: float
    n_exact: int


def approximate_attention_hybrid(query: torch.Tensor, full_key: torch.Tensor,
                                 full_value: torch.Tensor, summary: TorchSummary,
                                 sample_end: int, topk: int, samples: int,
                                 ranks: torch.Tensor | None = None,
                                 generator: torch.Generator | None = None) -> HeadResult:
    """One (sequence, query head) of a decode step: query [D] fp32, full_key /
    full_value [n_total, D] in the cache dtype.  ``ranks`` (int64 [samples]
    in [0, n_rest)) fixes the uniform draws; otherwise they come from
    ``torch.randint`` as in the reference's uniform mode."""
    n_total = int(full_key.shape[0])
    old_end = int(sample_end)
    scale = 1.0 / math.sqrt(full_key.shape[1])
    recent_scores = full_key[old_end:].float() @ query * scale
    recent_values = full_value[old_end:].float()

    guess = torch.log(summary.lengths_float) + summary.key_centroids @ query * scale
    chosen = torch.argsort(guess, descending=True, stable=True)[:topk]
    ranges = [summary.members[s:s + n] for s, n in
              zip(summary.starts[chosen].tolist(), summary.lengths_long[chosen].tolist())]
    exact_idx = torch.cat(ranges) if ranges else torch.zeros(0, dtype=torch.long)
    n_rest = old_end - int(exact_idx.numel())
    if n_rest > 0 and samples > 0:
        if ranks is None:
            ranks = torch.randint(n_rest, (samples,), generator=generator)
        sampled_idx = summary.members[rest_positions(summary, chosen, ranks.long())]
        log_proposal = torch.full((sampled_idx.numel(),), -math.log(n_rest),
                                  dtype=torch.float32)
    else:
        sampled_idx = torch.zeros(0, dtype=torch.long)
        log_proposal = torch.zeros(0, dtype=torch.float32)
    s_count = max(1, int(sampled_idx.numel()))

    exact_scores = full_key[exact_idx].float() @ query * scale
    sampled_scores = full_key[sampled_idx].float() @ query * scale
    sampled_log_weights = sampled_scores - log_proposal
    maximum = torch.cat((sampled_log_weights, exact_scores, recent_scores)).max()
    sampled_weights = torch.exp(sampled_log_weights - maximum) / s_count
    exact_weights = torch.exp(exact_scores - maximum)
    recent_weights = torch.exp(recent_scores - maximum)
    if sampled_idx.numel():
        normalized = torch.exp(sampled_log_weights - sampled_log_weights.max())
        ess = float((normalized.sum().square() / normalized.square().sum() / s_count).item())
    else:
        ess = 0.0
    numerator = (sampled_weights @ full_value[sampled_idx].float()
                 + exact_weights @ full_value[exact_idx].float()
                 + recent_weights @ recent_values)
    denominator = sampled_weights.sum() + exact_weights.sum() + recent_weights.sum()
    return HeadResult(numerator / denominator, ess, int(exact_idx.numel()))
