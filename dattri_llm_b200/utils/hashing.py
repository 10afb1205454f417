"""Content hashing of model inputs: the identity of a sample in the gradient store.

The digest is the reference's on-disk identity (``dattri_llm/utils/hashing.py``),
kept byte-for-byte so stores written by either framework resolve the same
samples: SHA-256 over, for each field in sorted key order, the UTF-8 key
followed by the field's raw C-contiguous bytes; padding is stripped first using
a 1-D ``attention_mask`` (fields of the mask's length keep the unmasked
positions, the mask itself is left out).  Lists, tuples and numeric scalars are
converted with ``torch.tensor`` so a raw ``dataset[i]`` hashes like its
collated tensor row.

What differs is the execution: :func:`hash_batch` moves every field of a batch
to the host once (one device-to-host copy per field instead of one per sample
and field) and hashes the per-sample byte slices from the host arrays, which
also lets the capture engine hash a batch on a side thread while the GPU runs.
"""

from __future__ import annotations

import hashlib
import warnings
from collections import Counter

import numpy as np
import torch

PAD_MASK_KEY = "attention_mask"


def _as_tensor(value: object) -> torch.Tensor | None:
    if isinstance(value, torch.Tensor):
        return value
    if isinstance(value, np.ndarray):
        return torch.from_numpy(value)
    if isinstance(value, (list, tuple, int, float, bool)):
        try:
            return torch.tensor(value)
        except (TypeError, ValueError, RuntimeError):
            return None
    return None


def _host_array(t: torch.Tensor) -> np.ndarray:
    t = t.detach()
    if t.device.type != "cpu":
        t = t.cpu()
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy()
    return t.contiguous().numpy()


def _strip(fields: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    mask = fields.get(PAD_MASK_KEY)
    if mask is None or mask.ndim != 1:
        return fields
    keep = mask.astype(bool)
    out = {}
    for key, arr in fields.items():
        if key == PAD_MASK_KEY:
            continue
        if arr.ndim >= 1 and arr.shape[0] == keep.shape[0]:
            arr = arr[keep]
        out[key] = arr
    return out


def _digest(fields: dict[str, np.ndarray]) -> str:
    h = hashlib.sha256()
    for key in sorted(fields):
        h.update(key.encode())
        h.update(np.ascontiguousarray(fields[key]).tobytes())
    return h.hexdigest()


def hash_sample(inputs: dict[str, object]) -> str:
    """SHA-256 content hash identifying **one sample** by its model inputs.

    Args:
        inputs: One sample's fields (e.g. what ``dataset[i]`` yields, or one row
            of a batch).  Tensors, numeric lists/tuples and numeric scalars are
            digested; other fields are skipped.

    Returns:
        64-character hex digest, independent of the batch the sample was padded in.

    Raises:
        ValueError: if no field is digestible.
    """
    fields: dict[str, np.ndarray] = {}
    for key, value in inputs.items():
        t = _as_tensor(value)
        if t is not None:
            fields[key] = _host_array(t)
    if not fields:
        raise ValueError(
            "hash_sample found no digestible field (tensor, numeric list/tuple or "
            f"numeric scalar) among keys {sorted(inputs)}",
        )
    fields = _strip(fields)
    return _digest(fields)


def _infer_batch_size(tensors: dict[str, torch.Tensor], inputs: dict) -> int:
    dims = [v.shape[0] for v in tensors.values()]
    if not dims:
        raise ValueError(
            "hash_batch could not infer a batch size: no non-scalar tensor field "
            f"among keys {sorted(inputs)}. Pass batch_size.",
        )
    counts = Counter(d for d in dims if d != 1)
    if not counts:
        return 1
    if len(counts) > 1:
        best = max(counts, key=lambda d: (counts[d], d))
        warnings.warn(
            f"hash_batch inferred batch_size={best} from fields with conflicting "
            f"leading dimensions { {k: v.shape[0] for k, v in tensors.items()} }; "
            "the disagreeing fields do not enter any sample's identity. Pass "
            "batch_size explicitly.",
            stacklevel=3,
        )
        return best
    return next(iter(counts))


def hash_batch(inputs: dict[str, object], batch_size: int | None = None) -> list[str]:
    """Per-sample content hashes of a **batched** input dict, in batch order.

    ``hash_batch(batch, B)[i] == hash_sample({k: v[i] for k, v in batch.items()})``
    over the batch-first fields.  Fields whose leading dimension is not the batch
    (broadcast ``position_ids``, packed ``cu_seqlens``) are skipped.

    Raises:
        ValueError: for a non-positive or un-inferable batch size, or when no
            batch-first field is left.
    """
    tensors = {
        k: v for k, v in inputs.items() if isinstance(v, torch.Tensor) and v.ndim > 0
    }
    if batch_size is None:
        batch_size = _infer_batch_size(tensors, inputs)
    elif batch_size < 1:
        raise ValueError(f"batch_size must be >= 1, got {batch_size}.")
    host: dict[str, np.ndarray | list] = {
        k: _host_array(v) for k, v in tensors.items() if v.shape[0] == batch_size
    }
    for k, v in inputs.items():
        if isinstance(v, (list, tuple)) and len(v) == batch_size and k not in host:
            host[k] = list(v)
    if not host:
        raise ValueError(
            f"hash_batch found no batch-first field (batch size {batch_size}) among "
            f"keys {sorted(inputs)}",
        )
    out = []
    for i in range(batch_size):
        fields: dict[str, np.ndarray] = {}
        for k, v in host.items():
            if isinstance(v, np.ndarray):
                fields[k] = v[i]
            else:
                t = _as_tensor(v[i])
                if t is not None:
                    fields[k] = _host_array(t)
        if not fields:
            raise ValueError("hash_batch: a sample has no digestible field")
        out.append(_digest(_strip(fields)))
    return out
