"""RWKV-4 checkpoint loader: a `.pth` state dict (the BlinkDL training
layout the reference loads through `rwkv.model.RWKV`, krunch/inference.py:
183-193) -> the step_ref weight dictionary RWKVModel takes
(scripts/rwkv4_step_ref.py:72-74,148-149: matrices [in, out]).

Transforms, as the third-party loader of rwkv==0.8.26 applies them for
RWKV-4 (its published loading rules, restated here):
* `emb.weight` is replaced by LayerNorm(emb, blocks.0.ln0) (eps 1e-5) and the
  ln0 parameters are dropped — the model then starts from ln1 of block 0;
* `*.time_mix_*`, `time_first`, `time_decay` are squeezed to [C];
  `time_decay` stays the raw log-decay (both WKV conventions of this library
  take it raw and form exp(time_decay) themselves);
* the five projection matrices of a block and `head.weight` are stored by the
  checkpoint as torch Linear weights [out, in] and are transposed to [in, out].
Everything is returned as float32 numpy arrays.
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np

_LINEAR = ("att.key.weight", "att.value.weight", "att.receptance.weight", "att.output.weight",
           "ffn.key.weight", "ffn.value.weight", "ffn.receptance.weight")

PILE_169M_FILE = "RWKV-4-Pile-169M-20220807-8023.pth"


def _f32(t) -> np.ndarray:
    if hasattr(t, "detach"):
        t = t.detach().float().cpu().numpy()
    return np.ascontiguousarray(np.asarray(t, dtype=np.float32))


def _layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    m = x.mean(axis=-1, keepdims=True, dtype=np.float64)
    v = ((x - m) ** 2).mean(axis=-1, keepdims=True, dtype=np.float64)
    return ((x - m) / np.sqrt(v + eps) * w + b).astype(np.float32)


def convert_state_dict(sd: dict) -> dict:
    """Checkpoint state dict (tensors or arrays) -> step_ref dict."""
    w = {k: _f32(v) for k, v in sd.items()}
    out: dict = {}
    if "blocks.0.ln0.weight" in w:
        out["emb.weight"] = _layer_norm(w["emb.weight"], w["blocks.0.ln0.weight"],
                                        w["blocks.0.ln0.bias"])
    else:
        out["emb.weight"] = w["emb.weight"]
    for k, v in w.items():
        if k == "emb.weight" or ".ln0." in k:
            continue
        if k == "head.weight" or any(k.endswith(s) for s in _LINEAR):
            out[k] = np.ascontiguousarray(v.T)
        elif ".time_" in k:
            out[k] = np.ascontiguousarray(v.reshape(-1))
        else:
            out[k] = v
    return out


def load_rwkv4_checkpoint(path: str | os.PathLike) -> dict:
    """Load a `.pth` RWKV-4 checkpoint (CPU, weights only) into the step_ref dict."""
    import torch
    sd = torch.load(str(path), map_location="cpu", weights_only=True)
    return convert_state_dict(sd)


def pretrained_path(model_dir: str | os.PathLike | None = None) -> Path | None:
    """The RWKV-4-Pile-169M checkpoint under $KRUNCH_MODEL_DIR, if present."""
    d = Path(model_dir or os.environ.get("KRUNCH_MODEL_DIR", "models"))
    p = d / PILE_169M_FILE
    return p if p.exists() else None
