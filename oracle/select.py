"""numpy restatement of the reference's YOLO26 selection (test infrastructure only).

Follows selection_flow.cpp:30-57 (score_key, float_bits, record order) and
:322-366 (packing); equal to verify_selection_flow.py ``reference()`` (:27-47),
which ranks by torch.argsort(descending=True, stable=True).  Adds the
``nan_last`` variant (NaN keys after -inf) that the config's wording asks for.
"""
from __future__ import annotations

import numpy as np

TRACE_NAMES = ("output", "class_max", "stage1_indices", "gathered_scores", "top_values",
               "stage2_indices", "anchor_indices", "labels")


def score_keys(bits: np.ndarray, nan_last: bool = False) -> np.ndarray:
    """selection_flow.cpp:30-35: 0 for NaN, 0x7fff for +-0, h for negatives,
    0x7fff - h for positives (smaller key ranks first)."""
    h = bits.astype(np.uint32)
    magnitude = h & 0x7FFF
    key = np.where(h & 0x8000, h, (~(h ^ 0x8000)) & 0xFFFF)
    key = np.where(magnitude == 0, 0x7FFF, key)
    key = np.where(magnitude > 0x7C00, 0xFFFF if nan_last else 0, key)
    return key.astype(np.uint32)


def float_bits(bits: np.ndarray) -> np.ndarray:
    """Exact fp16 -> fp32 widening on bits; NaNs keep sign/payload and are quieted
    (selection_flow.cpp:37-51)."""
    h = bits.astype(np.uint32)
    sign = (h & 0x8000) << 16
    exponent = (h >> 10) & 31
    mantissa = h & 1023
    out = np.where(exponent == 31,
                   sign | 0x7F800000 | (mantissa << 13) | np.where(mantissa != 0, 0x00400000, 0),
                   sign | ((exponent + 112) << 23) | (mantissa << 13))
    out = np.where((exponent == 0) & (mantissa == 0), sign, out)
    sub = (exponent == 0) & (mantissa != 0)
    if sub.any():
        m = mantissa[sub].astype(np.uint32)
        # normalise: shift until bit 10 is set
        shift = 10 - np.floor(np.log2(m)).astype(np.int64)
        e = 113 - shift
        m = (m << shift.astype(np.uint32)) & 1023
        out = out.copy()
        out[sub] = sign[sub] | (e.astype(np.uint32) << 23) | (m << 13)
    return out.astype(np.uint32)


def _stable_order(keys: np.ndarray) -> np.ndarray:
    """Indices sorted by (key, index): the reference's TileSort key*128+rank."""
    return np.argsort(keys, axis=-1, kind="stable")


_KEY_TABLES = {}


def _keys_of(bits: np.ndarray, nan_last: bool) -> np.ndarray:
    """score_keys through a 65,536-entry table built by score_keys itself (the same
    keys; fast on large score arrays)."""
    table = _KEY_TABLES.get(nan_last)
    if table is None:
        table = _KEY_TABLES[nan_last] = score_keys(np.arange(65536, dtype=np.uint32), nan_last)
    return table[bits.astype(np.uint16)]


def class_max(decoded_bits: np.ndarray, nan_last: bool = False, chunk: int = 64):
    """Stage 1 of the selection: per anchor, the first class with the smallest key
    (selection_max.h:74-79).  Returns (labels [B, A] int64, class_max [B, A] uint16),
    computed `chunk` images at a time."""
    bits = np.ascontiguousarray(decoded_bits, dtype=np.uint16)
    b, a, _ = bits.shape
    labels = np.zeros((b, a), np.int64)
    best = np.zeros((b, a), np.uint16)
    for i in range(0, b, chunk):
        scores = bits[i:i + chunk, :, 4:]
        if a and scores.shape[-1]:
            labels[i:i + chunk] = np.argmin(_keys_of(scores, nan_last), axis=-1)
            best[i:i + chunk] = np.take_along_axis(scores, labels[i:i + chunk, :, None], -1)[..., 0]
    return labels, best


def select(decoded_bits: np.ndarray, max_det: int, agnostic: bool = False,
           nan_last: bool = False, stage1=None):
    """decoded_bits: uint16 [B, A, 4+nc] (fp16 bit patterns, any layout).

    Returns the 8 trace stages of detection_select_trace (selection_flow.cpp:
    497-499) as numpy arrays: output [B,k,6] float32 bits as uint32, class_max
    [B,A] uint16, stage1_indices [B,k], gathered_scores [B,k|0,nc] uint16,
    top_values [B,k] uint16, stage2_indices [B,k|0], anchor_indices [B,k],
    labels [B,k].  ``stage1`` may pass class_max(decoded_bits, nan_last) computed
    once for several calls on the same scores."""
    bits = np.ascontiguousarray(decoded_bits, dtype=np.uint16)
    b, a, channels = bits.shape
    nc, k = channels - 4, min(max_det, a)
    scores = bits[..., 4:]
    labels_all, best = stage1 if stage1 is not None else class_max(bits, nan_last)
    first = _stable_order(_keys_of(best, nan_last))[:, :k] if a else np.zeros((b, 0), np.int64)
    if agnostic:
        top = np.take_along_axis(best, first, 1)
        label = np.take_along_axis(labels_all, first, 1)
        anchor = first
        gathered = np.zeros((b, 0, nc), np.uint16)
        second = np.zeros((b, 0), np.int64)
    else:
        gathered = np.take_along_axis(scores, first[..., None].repeat(nc, -1) if nc else first[..., None], 1) \
            if k else np.zeros((b, 0, nc), np.uint16)
        flat = gathered.reshape(b, k * nc)
        second = _stable_order(_keys_of(flat, nan_last))[:, :k]
        top = np.take_along_axis(flat, second, 1)
        label = second % nc
        anchor = np.take_along_axis(first, second // nc, 1)
    boxes = np.take_along_axis(bits[..., :4], anchor[..., None].repeat(4, -1), 1) if k else \
        np.zeros((b, 0, 4), np.uint16)
    out = np.zeros((b, k, 6), np.uint32)
    out[..., :4] = float_bits(boxes)
    out[..., 4] = float_bits(top)
    out[..., 5] = label.astype(np.float32).view(np.uint32)
    return dict(zip(TRACE_NAMES, (out, best, first.astype(np.int64), gathered,
                                  top.astype(np.uint16), second.astype(np.int64),
                                  anchor.astype(np.int64), label.astype(np.int64))))
