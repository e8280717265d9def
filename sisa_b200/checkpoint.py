"""Weight I/O in the reference's formats (mirrors src/sisa/checkpoint.py of tlstngud/sisa).

Two on-disk formats are read, and the second is written, byte-compatible with the reference so that a
file made by either package loads into the other:

* **Paper training checkpoints** (checkpoint.py:1-10, 156-183): a ``torch.save`` file whose
  ``"model"`` (or ``"state_dict"``) entry is a state dict, or a bare state dict. Its attention
  parameters sit directly under ``layers.{i}.`` (``layers.0.W_Q.weight``), modules compiled during
  training carry an ``_orig_mod`` name part (``layers.0.ffn._orig_mod.w_gate.weight``), and a DDP
  wrapper adds a leading ``module.``. Everything else in the file (optimizer, scheduler, stored
  training config) is dropped unread.
* **Pretrained directories** (checkpoint.py:186-250): ``config.json`` holding
  :meth:`SISAConfig.to_dict` and the weights in ``model.safetensors`` (metadata ``{"format": "pt"}``)
  or ``pytorch_model.bin``.

The parameter names of :class:`sisa_b200.SISAForCausalLM` are the reference's, so a converted state
dict loads strictly. Models come back on the CPU in eval mode; move them with ``.to("cuda")``.
"""
from __future__ import annotations

import json
import pickle
from pathlib import Path
from typing import TYPE_CHECKING, Any, Mapping

import torch
from torch import Tensor

from .config import SISAConfig

if TYPE_CHECKING:  # pragma: no cover
    from .modeling import SISAForCausalLM

__all__ = ["convert_state_dict", "infer_config_from_state_dict", "load_paper_checkpoint", "save_pretrained",
           "from_pretrained", "CONFIG_NAME", "SAFETENSORS_NAME", "TORCH_WEIGHTS_NAME"]

CONFIG_NAME = "config.json"
SAFETENSORS_NAME = "model.safetensors"
TORCH_WEIGHTS_NAME = "pytorch_model.bin"

#: Per-layer attention parameters that the paper code stores directly under ``layers.{i}``
#: (checkpoint.py:41); this package keeps them under ``layers.{i}.attn``.
ATTN_PARAM_NAMES = frozenset({"W_Q", "W_K", "W_V", "W_O", "W_B", "W_C", "alpha_proj", "theta_proj",
                              "forget_proj", "lambda_raw"})
_COMPILE_PART = "_orig_mod"      # torch.compile's wrapper attribute
_DDP_PART = "module"             # DistributedDataParallel's wrapper attribute


def _package_key(key: str) -> str:
    """One checkpoint key in this package's naming (checkpoint.py:46-79).

    Leading wrapper names (``module``, ``_orig_mod``, in any order and number) and every interior
    ``_orig_mod`` part are dropped; an attention parameter directly under ``layers.{i}`` moves under
    ``layers.{i}.attn``. A key already in this package's naming comes back unchanged.
    """
    parts = key.split(".")
    start = 0
    while start < len(parts) - 1 and parts[start] in (_DDP_PART, _COMPILE_PART):
        start += 1
    parts = [p for p in parts[start:] if p != _COMPILE_PART]
    if len(parts) >= 3 and parts[0] == "layers" and parts[1].isdecimal() and parts[2] in ATTN_PARAM_NAMES:
        parts.insert(2, "attn")
    return ".".join(parts)


def convert_state_dict(state_dict: Mapping[str, Tensor]) -> dict[str, Tensor]:
    """Rename a paper (or already converted) state dict to this package's parameter names.

    Idempotent. Raises ``ValueError`` when two keys of the input map to the same name.
    """
    out: dict[str, Tensor] = {}
    for key, value in state_dict.items():
        name = _package_key(key)
        if name in out:
            raise ValueError(f"two checkpoint keys map to {name!r}")
        out[name] = value
    return out


def _layer_index(key: str) -> int | None:
    parts = key.split(".", 2)
    if len(parts) == 3 and parts[0] == "layers" and parts[1].isdecimal():
        return int(parts[1])
    return None


def infer_config_from_state_dict(state_dict: Mapping[str, Tensor], **overrides: Any) -> SISAConfig:
    """The model shape read from tensor shapes alone (checkpoint.py:82-106).

    ``vocab_size, d_model`` come from ``embed.weight``, ``n_head`` from ``lambda_raw``, ``d_state``
    from the rows of ``W_B`` per head, ``d_ff`` from ``ffn.w_gate`` (a stored training config may name
    a different, nominal width) and ``n_layer`` from the layer indices, which must run 0..n-1.
    ``overrides`` may set any other :class:`SISAConfig` field; naming a shape field is a
    ``ValueError``.
    """
    sd = convert_state_dict(state_dict)
    needed = ("embed.weight", "layers.0.attn.lambda_raw", "layers.0.attn.W_B.weight", "layers.0.ffn.w_gate.weight")
    for name in needed:
        if name not in sd:
            raise ValueError(f"not a SISA state dict: missing {name!r}")
    vocab_size, d_model = sd["embed.weight"].shape
    n_head = sd["layers.0.attn.lambda_raw"].numel()
    state_rows = sd["layers.0.attn.W_B.weight"].shape[0]
    d_ff = sd["layers.0.ffn.w_gate.weight"].shape[0]
    layers = sorted({i for i in map(_layer_index, sd) if i is not None})
    if layers != list(range(len(layers))):
        raise ValueError(f"layer indices are not contiguous: {layers}")
    if state_rows % n_head:
        raise ValueError(f"W_B has {state_rows} rows, not a multiple of n_head={n_head}")
    shape = {"vocab_size": int(vocab_size), "d_model": int(d_model), "n_layer": len(layers),
             "n_head": int(n_head), "d_ff": int(d_ff), "d_state": int(state_rows // n_head)}
    fixed = sorted(shape.keys() & overrides.keys())
    if fixed:
        raise ValueError(f"shape fields {fixed} are read from the weights and cannot be overridden")
    return SISAConfig(**shape, **overrides)


def _model_without_init(config: SISAConfig) -> "SISAForCausalLM":
    """A model whose parameters are allocated on the CPU but not initialised: the weights that are
    loaded next overwrite every one of them."""
    from .modeling import SISAForCausalLM

    with torch.device("meta"):
        model = SISAForCausalLM(config)
    return model.to_empty(device="cpu")


def _load_exact(model: torch.nn.Module, state_dict: Mapping[str, Tensor]) -> None:
    """Strict load: every model key present with its shape and nothing else, else ValueError listing the
    first few offending keys (missing / unexpected / shape mismatch)."""
    want = {k: tuple(t.shape) for k, t in model.state_dict().items()}
    have = {k: tuple(t.shape) for k, t in state_dict.items()}
    missing, unexpected = sorted(want.keys() - have.keys()), sorted(have.keys() - want.keys())
    if missing or unexpected:
        raise ValueError(f"the state dict does not fit the model: {len(missing)} missing keys {missing[:8]}, "
                         f"{len(unexpected)} unexpected keys {unexpected[:8]}")
    wrong = [(k, have[k], shape) for k, shape in want.items() if have[k] != shape]
    if wrong:
        raise ValueError(f"shape mismatch, as (key, checkpoint shape, model shape): {wrong[:8]}")
    model.load_state_dict(state_dict, strict=True)


def _weights_of(obj: Any) -> dict[str, Tensor]:
    """The state dict inside a loaded checkpoint object (checkpoint.py:132-140)."""
    if isinstance(obj, Mapping):
        for entry in ("model", "state_dict"):
            inner = obj.get(entry)
            if isinstance(inner, Mapping):
                return dict(inner)
        if obj and all(isinstance(v, Tensor) for v in obj.values()):
            return dict(obj)
    raise ValueError("checkpoint holds neither a 'model' state dict nor a plain state dict")


def _read_torch_file(path: Path, weights_only: bool) -> Any:
    """``torch.load`` to the CPU. Files in torch's zip format are memory-mapped (tensors are read on first
    use); older pickle-only files cannot be mapped and are read whole. With ``weights_only`` a file that
    needs arbitrary Python objects raises UnpicklingError naming the ``trust_pickle`` flag."""
    with open(path, "rb") as f:
        zip_format = f.read(4) == b"PK\x03\x04"
    try:
        return torch.load(path, map_location="cpu", mmap=zip_format, weights_only=weights_only)
    except pickle.UnpicklingError as err:
        raise pickle.UnpicklingError(
            f"{err}\n{path} stores Python objects beyond tensors, which the safe loader refuses; load it with "
            "trust_pickle=True only if you trust where the file came from.") from None


def load_paper_checkpoint(path: str | Path, *, trust_pickle: bool = False, dtype: torch.dtype | None = None,
                          **config_overrides: Any) -> "SISAForCausalLM":
    """Load a training checkpoint of the paper code (checkpoint.py:156-183).

    The file is read with ``weights_only=True`` unless ``trust_pickle=True`` (only for trusted files);
    a file that then needs arbitrary objects raises ``pickle.UnpicklingError`` naming the flag. The
    architecture comes from the tensor shapes, ``config_overrides`` set non-shape fields (for example
    ``attn_impl``), and the load is strict. ``dtype`` casts the model afterwards; ``lambda_raw`` stays
    fp32. Returns the model on the CPU in eval mode.
    """
    obj = _read_torch_file(Path(path), weights_only=not trust_pickle)
    weights = convert_state_dict(_weights_of(obj))
    del obj
    model = _model_without_init(infer_config_from_state_dict(weights, **config_overrides))
    _load_exact(model, weights)
    if dtype is not None:
        model.to(dtype)
    return model.eval()


def save_pretrained(model: torch.nn.Module, path: str | Path, *, safe_serialization: bool = True) -> None:
    """Write ``config.json`` and the weights into directory ``path`` (checkpoint.py:186-212).

    The weights go to ``model.safetensors`` when ``safe_serialization`` is set and ``safetensors`` is
    importable, else to ``pytorch_model.bin``; a weights file of the other format already in ``path``
    is deleted, so that :func:`from_pretrained` cannot read stale weights.
    """
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / CONFIG_NAME).write_text(json.dumps(model.config.to_dict(), indent=2) + "\n", encoding="utf-8")
    tensors = {k: v.detach().to("cpu").contiguous() for k, v in model.state_dict().items()}
    save_file = None
    if safe_serialization:
        try:
            from safetensors.torch import save_file
        except ImportError:
            save_file = None
    if save_file is not None:
        save_file(tensors, str(path / SAFETENSORS_NAME), metadata={"format": "pt"})
        stale = path / TORCH_WEIGHTS_NAME
    else:
        torch.save(tensors, path / TORCH_WEIGHTS_NAME)
        stale = path / SAFETENSORS_NAME
    stale.unlink(missing_ok=True)


def from_pretrained(path: str | Path, *, dtype: torch.dtype | None = None,
                    **config_overrides: Any) -> "SISAForCausalLM":
    """Load a directory written by :func:`save_pretrained` of this package or of the reference
    (checkpoint.py:215-250). ``config_overrides`` replace fields of the stored config. Returns the
    model on the CPU in eval mode.
    """
    path = Path(path)
    if not path.is_dir():
        raise ValueError(f"{path} is not a directory written by save_pretrained "
                         "(use load_paper_checkpoint for training checkpoints)")
    config = SISAConfig.from_dict(json.loads((path / CONFIG_NAME).read_text(encoding="utf-8")),
                                  **config_overrides)
    if (path / SAFETENSORS_NAME).exists():
        try:
            from safetensors.torch import load_file
        except ImportError:
            raise ImportError(f"{path / SAFETENSORS_NAME} needs the 'safetensors' package") from None
        weights = load_file(str(path / SAFETENSORS_NAME))
    elif (path / TORCH_WEIGHTS_NAME).exists():
        weights = torch.load(path / TORCH_WEIGHTS_NAME, map_location="cpu", weights_only=True)
    else:
        raise FileNotFoundError(f"no {SAFETENSORS_NAME} or {TORCH_WEIGHTS_NAME} in {path}")
    model = _model_without_init(config)
    _load_exact(model, convert_state_dict(weights))
    if dtype is not None:
        model.to(dtype)
    return model.eval()
