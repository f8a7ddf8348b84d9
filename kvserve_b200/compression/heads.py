"""Head-importance scores, low/high precision head selection and the
Rademacher sign vectors shared by every compression path.

* Scores: a ``[layers, kv_heads]`` table (DuoAttention retrieval scores).  The
  tables shipped in ``scores/`` are the published per-model measurements the
  reference uses (kvserve_v1/compression/config/duo_config/*.csv); they are
  data, kept identical so that head selection — and therefore the section
  order of every payload — matches the reference.  Models without a table get
  deterministic pseudo-scores from a seeded generator.
* Selection (kvserve_v1/compression/quantizer/kvserve_quantizer.py:57-68):
  the ``round(N * hybrid_ratio)`` lowest-scoring (layer, head) pairs of the
  whole model are low precision; with ``split_type="layer"`` the last
  ``round(0.33 * L)`` layers are low precision.  TP ranks slice their heads
  (kvserve_quantizer.py:76-103).
* Signs (kvserve_v1/compression/transformer/hadamard_func.py:33-159): head
  ``h`` of layer ``l`` uses seed ``base ^ (l << 16) ^ h`` and
  ``torch.randint(0, 2, (D,), generator=cpu_generator, dtype=int8)`` mapped to
  {-1, +1}.  The generator call is kept as is: it is what makes the signs —
  and so the transformed values — identical on both ends and with the
  reference.
"""
from __future__ import annotations

import functools
import os
from pathlib import Path
from typing import Optional

import numpy as np
import torch

_SCORES_DIR = Path(__file__).parent / "scores"


def _model_basename(model_name: str) -> str:
    return model_name.strip("/").split("/")[-1]


def load_scores_file(path: str | os.PathLike) -> torch.Tensor:
    """Load a ``[layers, kv_heads]`` score table from csv/npy/pt/json."""
    p = Path(path)
    suffix = p.suffix.lower()
    if suffix == ".csv":
        arr = np.loadtxt(p, delimiter=",", dtype=np.float32, ndmin=2)
    elif suffix == ".npy":
        arr = np.load(p).astype(np.float32)
    elif suffix == ".pt":
        arr = torch.load(p, map_location="cpu").float().numpy()
    elif suffix == ".json":
        import json
        arr = np.asarray(json.loads(p.read_text()), dtype=np.float32)
    else:
        raise ValueError(f"unsupported score file: {p}")
    if arr.ndim != 2:
        raise ValueError(f"score table must be 2-D [layers, kv_heads], got {arr.shape}")
    return torch.from_numpy(np.ascontiguousarray(arr))


def synthetic_scores(num_layers: int, num_kv_heads: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator(device="cpu")
    g.manual_seed(0x5C0DE ^ seed ^ (num_layers << 8) ^ num_kv_heads)
    return torch.rand((num_layers, num_kv_heads), generator=g, dtype=torch.float32)


@functools.lru_cache(maxsize=32)
def _cached_scores(model_name: str, num_layers: int, num_kv_heads: int) -> torch.Tensor:
    base = _model_basename(model_name) if model_name else ""
    for cand in (_SCORES_DIR / f"{base}_scores.csv", Path.cwd() / f"{base}_scores.csv", Path(f"{base}_scores.csv")):
        if base and cand.exists():
            t = load_scores_file(cand)
            if num_layers <= 0 or (t.shape[0] == num_layers and (num_kv_heads <= 0 or t.shape[1] == num_kv_heads)):
                return t
    if num_layers <= 0 or num_kv_heads <= 0:
        raise FileNotFoundError(f"no head-score table for model {model_name!r}")
    return synthetic_scores(num_layers, num_kv_heads)


def get_scores(model_name: Optional[str], num_layers: int = 0, num_kv_heads: int = 0,
               score_path: Optional[str] = None) -> torch.Tensor:
    """Score table for a model (shipped table, explicit file, or synthetic)."""
    if score_path:
        return load_scores_file(score_path)
    return _cached_scores(model_name or "", num_layers, num_kv_heads).clone()


def low_precision_mask(scores: torch.Tensor, hybrid_ratio: float, split_type: str = "head") -> torch.Tensor:
    """Boolean ``[layers, kv_heads]`` mask of low-precision heads."""
    layers, heads = scores.shape
    mask = torch.zeros((layers, heads), dtype=torch.bool)
    if split_type == "head":
        n_low = round(scores.numel() * hybrid_ratio)
        idx = torch.argsort(scores.flatten())[:n_low]
        mask.view(-1)[idx] = True
    elif split_type == "layer":
        n_low_layers = round(layers * 0.33)
        if n_low_layers > 0:
            mask[-n_low_layers:, :] = True
    else:
        raise ValueError(f"split_type must be 'head' or 'layer', got {split_type!r}")
    return mask


def tp_slice_mask(mask: torch.Tensor, local_heads: int, tp_rank: int, tp_size: int) -> torch.Tensor:
    """Columns of ``mask`` owned by one TP rank (replicated KV heads when
    ``tp_size > kv_heads``: rank r owns head ``r * kv_heads // tp_size``)."""
    total = mask.shape[1]
    if total == local_heads:
        return mask
    if tp_size > total and local_heads == 1:
        head = tp_rank * total // tp_size
        return mask[:, head:head + 1]
    if total % local_heads != 0 or total // local_heads != tp_size:
        raise ValueError(f"TP mismatch: mask heads={total}, local heads={local_heads}, tp_size={tp_size}")
    start = tp_rank * local_heads
    return mask[:, start:start + local_heads]


def section_orders(mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per layer: head order with low heads first (each group ascending, as
    boolean-mask indexing keeps order) and the number of low heads."""
    layers, heads = mask.shape
    order = torch.empty((layers, heads), dtype=torch.int32)
    n_low = torch.empty(layers, dtype=torch.int32)
    ar = torch.arange(heads, dtype=torch.int32)
    for l in range(layers):
        m = mask[l]
        low, high = ar[m], ar[~m]
        order[l] = torch.cat([low, high])
        n_low[l] = low.numel()
    return order, n_low


@functools.lru_cache(maxsize=4096)
def _signs_one(seed: int, head_dim: int) -> torch.Tensor:
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    s = torch.randint(0, 2, (head_dim,), generator=gen, dtype=torch.int8)
    return s.float().mul_(2).sub_(1)


def head_seed(base_seed: int, layer: int, head: int) -> int:
    return (int(base_seed) ^ (int(layer) << 16) ^ int(head)) & 0xFFFFFFFFFFFFFFFF


def rademacher_signs(base_seed: int, layer: int, num_heads: int, head_dim: int,
                     head_offset: int = 0) -> torch.Tensor:
    """``[num_heads, head_dim]`` fp32 ±1 signs; ``head_offset`` is the global
    index of local head 0 (tensor parallel shards keep global seeds)."""
    return torch.stack([_signs_one(head_seed(base_seed, layer, head_offset + h), head_dim)
                        for h in range(num_heads)])


def pack_sign_bits(signs: torch.Tensor) -> torch.Tensor:
    """``[..., D]`` ±1 -> int32 ``[..., D/32]`` with bit ``d % 32`` of word
    ``d // 32`` set where the sign is negative."""
    d = signs.shape[-1]
    if d % 32:
        raise ValueError("head_dim must be a multiple of 32")
    neg = (signs < 0).to(torch.int64).reshape(*signs.shape[:-1], d // 32, 32)
    weights = (torch.ones(32, dtype=torch.int64) << torch.arange(32, dtype=torch.int64))
    words = (neg * weights).sum(-1)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words)
    return words.to(torch.int32)
