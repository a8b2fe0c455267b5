"""Checkpoint / resume of the runtime's device state: every tensor a class
names in ``_state_tensors()`` (its SoA fields, value nodes, global-state
records) plus the scalars of ``_state_meta()``, written as one ``.npz`` file.
Loading copies each array into the existing tensor of an object built the
same way (same sizes and layout), so a resumed run continues bit for bit.
The reference has no serialisation; this is an addition."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

FORMAT = "plastix-b200-checkpoint-1"


def save_state(obj, path) -> None:
    tensors = obj._state_tensors()
    meta = {"format": FORMAT, "class": type(obj).__name__,
            "fields": {k: [str(t.dtype), list(t.shape)] for k, t in tensors.items()}}
    meta.update(obj._state_meta() if hasattr(obj, "_state_meta") else {})
    arrays = {k: t.detach().cpu().numpy() for k, t in tensors.items()}
    with open(Path(path), "wb") as f:
        np.savez(f, __meta__=np.array(json.dumps(meta)), **arrays)


def load_state(obj, path) -> dict:
    with np.load(Path(path), allow_pickle=False) as z:
        meta = json.loads(str(z["__meta__"]))
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path}: not a {FORMAT} file")
        if meta.get("class") != type(obj).__name__:
            raise ValueError(f"{path}: written by {meta.get('class')}, not {type(obj).__name__}")
        tensors = obj._state_tensors()
        if set(tensors) != set(meta["fields"]):
            raise ValueError(f"{path}: fields {sorted(meta['fields'])} differ from "
                             f"{sorted(tensors)}")
        for k, t in tensors.items():
            a = z[k]
            if list(a.shape) != list(t.shape) or str(t.dtype) != meta["fields"][k][0]:
                raise ValueError(f"{path}: field {k} is {meta['fields'][k]}, expected "
                                 f"{[str(t.dtype), list(t.shape)]}")
        for k, t in tensors.items():
            t.copy_(torch.from_numpy(np.ascontiguousarray(z[k])))
    if hasattr(obj, "_load_meta"):
        obj._load_meta(meta)
    return meta
