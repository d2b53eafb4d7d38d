"""Label readout of a logits row: `Readout::Label` of omg-core
(crates/omg-core/src/readout.rs:124-147) with its numeric helpers
(crates/omg-core/src/math.rs:5-17).

A branch's answer row holds `vocab` logits (``Want.LOGITS``); the k option
labels are single tokens, their logits are the option logits, the
probabilities are the softmax of those over a temperature, in f64, and the
candidate mass is how much of the whole row's probability the labels hold,
exp(lse(labels) - lse(row)).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Distribution:
    """readout.rs `Distribution` for the label readout."""
    logits: np.ndarray          # f32 option logits, label order
    probs: np.ndarray           # f64 softmax(logits / temperature)
    candidate_mass: float       # exp(lse(labels) - lse(row))


def softmax(z, temperature: float = 1.0) -> np.ndarray:
    """math.rs:5-11: softmax of z / temperature in f64 after subtracting the
    f32 maximum; the temperature is floored at 1e-6."""
    z = np.asarray(z, dtype=np.float32)
    t = float(max(np.float32(temperature), np.float32(1e-6)))
    m = float(z.max())
    e = np.exp((z.astype(np.float64) - m) / t)
    return e / e.sum()


def log_sum_exp(z) -> float:
    """math.rs:13-17, in f64 around the f32 maximum."""
    z = np.asarray(z, dtype=np.float32)
    m = float(z.max())
    return m + float(np.log(np.exp(z.astype(np.float64) - m).sum()))


def label_distribution(row, label_ids, temperature: float = 1.0) -> Distribution:
    """readout.rs:130-147 (Readout::Label): `row` one answer row of logits,
    `label_ids` the option labels' token ids in option order."""
    row = np.asarray(row, dtype=np.float32)
    ids = np.asarray(label_ids, dtype=np.int64)
    if ids.size == 0:
        raise ValueError("no option labels")
    if ids.min() < 0 or ids.max() >= row.size:
        raise ValueError("label id outside the vocabulary")
    logits = row[ids]
    return Distribution(logits=logits, probs=softmax(logits, temperature),
                        candidate_mass=float(np.exp(log_sum_exp(logits) - log_sum_exp(row))))
