"""Torque artifacts: a directory with ``manifest.json`` and an npz of fused
attention weights, as written by the reference (src/torque_mlx/artifact.py).

The on-disk format is the reference's, so artifacts move between the two
implementations: manifest keys, the ``torque-mlx-artifact`` / version-1 tag,
the runtime-config and codebook objects, and the npz member names listed in
``weight_names``.  What this module needs from an artifact is the runtime
configuration and the two codebooks, from which ``build_cache()`` makes the
GPU cache (artifact.py:157-162); it also writes artifacts and folds weights so
a model converted here reads back in the reference.

The manifest is handled through one field table (``_FIELDS``): each entry
names the JSON key, whether it is required, its default and how a value is
decoded and encoded.  Parsing, validation and writing all walk that table.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field, replace
from pathlib import Path
from typing import Any, Callable, Mapping

import numpy as np

from .cache import TorqueKVCache
from .config import RotationMode, TorqueConfig
from .conversion import FusedAttentionWeights, fuse_attention_weights
from .quantization import Codebook, build_gaussian_codebook
from .rotation import RotationSpec

FORMAT_TAG = "torque-mlx-artifact"
FORMAT_VERSION = 1
MANIFEST_NAME = "manifest.json"
WEIGHTS_NAME = "weights.npz"
PROJECTIONS = ("w_q", "w_k", "w_v", "w_o")


def _plain(v: Any) -> Any:
    """JSON-safe copy: numpy scalars become Python numbers, tuples lists."""
    if isinstance(v, Mapping):
        return {str(k): _plain(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_plain(x) for x in v]
    return v.item() if isinstance(v, np.generic) else v


# runtime_config object <-> TorqueConfig (the key set is part of the format)
_CONFIG_KEYS: tuple[tuple[str, Callable[[Any], Any]], ...] = (
    ("bit_width", int), ("head_dim", int), ("num_layers", int), ("kv_heads", int),
    ("fused_weights", bool), ("rotation_mode", lambda v: RotationMode(str(v))), ("rotation_seed", int),
)


def _config_in(obj: Any) -> TorqueConfig:
    if not isinstance(obj, Mapping):
        raise ValueError("manifest runtime_config is not a JSON object")
    absent = [k for k, _ in _CONFIG_KEYS if k not in obj]
    if absent:
        raise ValueError(f"manifest runtime_config lacks {', '.join(absent)}")
    return TorqueConfig(**{k: conv(obj[k]) for k, conv in _CONFIG_KEYS})


def _config_out(cfg: TorqueConfig) -> dict[str, Any]:
    out = {k: getattr(cfg, k) for k, _ in _CONFIG_KEYS}
    out["rotation_mode"] = cfg.rotation_mode.value
    return out


def _names_in(obj: Any) -> dict[str, str]:
    names = {str(k): str(v) for k, v in dict(obj or {}).items()}
    return names or {p: p for p in PROJECTIONS}


_REQUIRED = object()

# (json key, attribute, default or _REQUIRED, decode, encode); default None =
# absent keys decode from None
_FIELDS: tuple[tuple[str, str, Any, Callable, Callable], ...] = (
    ("format_name", "format_name", FORMAT_TAG, str, str),
    ("format_version", "format_version", FORMAT_VERSION, int, int),
    ("model_name", "model_name", _REQUIRED, str, str),
    ("architecture", "architecture", _REQUIRED, str, str),
    ("source_format", "source_format", _REQUIRED, str, str),
    ("runtime_config", "runtime_config", _REQUIRED, _config_in, _config_out),
    ("weights_file", "weights_file", WEIGHTS_NAME, str, str),
    ("weight_names", "weight_names", None, _names_in, dict),
    ("key_codebook", "key_codebook", _REQUIRED, lambda v: Codebook.from_dict(dict(v)), lambda c: c.to_dict()),
    ("value_codebook", "value_codebook", _REQUIRED, lambda v: Codebook.from_dict(dict(v)), lambda c: c.to_dict()),
    ("extra_metadata", "extra_metadata", None, lambda v: _plain(dict(v or {})), _plain),
)


@dataclass(frozen=True)
class TorqueArtifactManifest:
    """Parsed ``manifest.json``; the runtime config must use fused weights
    (an artifact stores projections with the rotation folded in)."""

    model_name: str
    architecture: str
    source_format: str
    runtime_config: TorqueConfig
    key_codebook: Codebook
    value_codebook: Codebook
    weights_file: str = WEIGHTS_NAME
    format_name: str = FORMAT_TAG
    format_version: int = FORMAT_VERSION
    weight_names: dict[str, str] = field(default_factory=lambda: {p: p for p in PROJECTIONS})
    extra_metadata: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.format_name != FORMAT_TAG:
            raise ValueError(f"not a torque artifact: format_name {self.format_name!r}")
        if self.format_version != FORMAT_VERSION:
            raise ValueError(f"artifact format version {self.format_version} is not supported "
                             f"(this build reads version {FORMAT_VERSION})")
        self.runtime_config.validate()
        if not self.runtime_config.fused_weights:
            raise ValueError("an artifact's runtime_config must have fused_weights = true")
        for p in PROJECTIONS:
            if p not in self.weight_names:
                raise ValueError(f"manifest weight_names has no entry for {p}")

    @classmethod
    def from_dict(cls, payload: Mapping[str, Any]) -> "TorqueArtifactManifest":
        absent = [key for key, _, default, _, _ in _FIELDS if default is _REQUIRED and key not in payload]
        if absent:
            raise ValueError(f"manifest lacks required key(s): {', '.join(absent)}")
        kwargs = {}
        for key, attr, default, decode, _ in _FIELDS:
            if key in payload:
                kwargs[attr] = decode(payload[key])
            elif default is None:
                kwargs[attr] = decode(None)
        return cls(**kwargs)

    def to_dict(self) -> dict[str, Any]:
        out = {key: encode(getattr(self, attr)) for key, attr, _, _, encode in _FIELDS}
        out["variant_id"] = self.runtime_config.variant_id
        return out


@dataclass(frozen=True)
class TorqueArtifact:
    manifest: TorqueArtifactManifest
    fused_weights: FusedAttentionWeights

    runtime_config = property(lambda self: self.manifest.runtime_config)
    key_codebook = property(lambda self: self.manifest.key_codebook)
    value_codebook = property(lambda self: self.manifest.value_codebook)

    def build_cache(self, **cache_kwargs) -> TorqueKVCache:
        """The packed GPU cache for this artifact: its runtime config and both
        codebooks (artifact.py:157-162).  Extra keywords (``batch_size``,
        ``initial_capacity``, ``decode_mode``, ...) go to the cache."""
        return TorqueKVCache(config=self.runtime_config, key_codebook=self.key_codebook,
                             value_codebook=self.value_codebook, **cache_kwargs)

    def save(self, directory: str | Path, *, force: bool = False) -> Path:
        """Write the manifest (sorted keys, indent 2) and the npz; a non-empty
        directory is only replaced with ``force``."""
        target = Path(directory)
        if not force and target.is_dir() and next(target.iterdir(), None) is not None:
            raise FileExistsError(f"{target} already holds files; use force=True to write the artifact there")
        target.mkdir(parents=True, exist_ok=True)
        (target / MANIFEST_NAME).write_text(json.dumps(self.manifest.to_dict(), indent=2, sort_keys=True),
                                            encoding="utf-8")
        names = self.manifest.weight_names
        np.savez_compressed(target / self.manifest.weights_file,
                            **{names[p]: getattr(self.fused_weights, p) for p in PROJECTIONS})
        return target

    def summary(self) -> dict[str, Any]:
        m = self.manifest

        def book(c: Codebook) -> dict[str, Any]:
            return {"name": c.name, "bit_width": c.bit_width, "centroid_count": int(c.centroids.size)}

        return {
            "format_name": m.format_name, "format_version": m.format_version, "model_name": m.model_name,
            "architecture": m.architecture, "source_format": m.source_format,
            "variant_id": m.runtime_config.variant_id, "weights_file": m.weights_file,
            "runtime_config": _config_out(m.runtime_config),
            "weight_shapes": {p: list(np.shape(getattr(self.fused_weights, p))) for p in PROJECTIONS},
            "key_codebook": book(m.key_codebook), "value_codebook": book(m.value_codebook),
            "extra_metadata": _plain(m.extra_metadata),
        }

    @classmethod
    def load(cls, directory: str | Path) -> "TorqueArtifact":
        root = Path(directory)
        mpath = root / MANIFEST_NAME
        if not mpath.is_file():
            raise FileNotFoundError(f"no {MANIFEST_NAME} in {root}")
        manifest = TorqueArtifactManifest.from_dict(json.loads(mpath.read_text(encoding="utf-8")))
        wpath = root / manifest.weights_file
        if not wpath.is_file():
            raise FileNotFoundError(f"weights file {wpath} named by the manifest is missing")
        with np.load(wpath) as z:
            w = {p: np.asarray(z[manifest.weight_names[p]], dtype=np.float32) for p in PROJECTIONS}
        return cls(manifest=manifest,
                   fused_weights=FusedAttentionWeights(**w, rotation_seed=manifest.runtime_config.rotation_seed))


def load_torque_artifact(directory: str | Path) -> TorqueArtifact:
    return TorqueArtifact.load(directory)


def build_torque_artifact(*, model_name: str, architecture: str, source_format: str, config: TorqueConfig,
                          w_q, w_k, w_v, w_o, rotation: RotationSpec | None = None,
                          key_codebook: Codebook | None = None, value_codebook: Codebook | None = None,
                          extra_metadata: Mapping[str, Any] | None = None) -> TorqueArtifact:
    """Fold the rotation into the four projections (on the GPU, exact
    rotation kernel) and describe them with a fused-weights runtime config.
    Default codebooks follow the cache's seeds (K: rotation_seed, V: + 1)."""
    cfg = replace(config, fused_weights=True)
    rot = rotation or RotationSpec.from_seed(head_dim=cfg.head_dim, seed=cfg.rotation_seed)
    kb = key_codebook or build_gaussian_codebook(cfg.bit_width, seed=cfg.rotation_seed)
    vb = value_codebook or build_gaussian_codebook(cfg.bit_width, seed=cfg.rotation_seed + 1)
    fused = fuse_attention_weights(w_q=w_q, w_k=w_k, w_v=w_v, w_o=w_o, rotation=rot)
    meta: dict[str, Any] = {"input_dim": int(np.shape(w_q)[1]), "output_dim": int(np.shape(w_o)[0])}
    meta.update(_plain(dict(extra_metadata or {})))
    manifest = TorqueArtifactManifest(model_name=model_name, architecture=architecture,
                                      source_format=source_format, runtime_config=cfg, key_codebook=kb,
                                      value_codebook=vb, extra_metadata=meta)
    return TorqueArtifact(manifest=manifest, fused_weights=fused)


def convert_npz_checkpoint(*, input_path: str | Path, output_dir: str | Path, model_name: str | None,
                           architecture: str, source_format: str, bit_width: int, num_layers: int, kv_heads: int,
                           rotation_seed: int, head_dim: int | None = None, key_codebook: Codebook | None = None,
                           value_codebook: Codebook | None = None, force: bool = False) -> TorqueArtifact:
    """npz holding w_q / w_k / w_v / w_o -> artifact directory.  head_dim
    defaults to w_q's output dimension."""
    with np.load(input_path) as z:
        absent = [p for p in PROJECTIONS if p not in z.files]
        if absent:
            raise ValueError(f"{input_path} lacks the projection array(s) {', '.join(absent)}")
        w = {p: np.asarray(z[p]) for p in PROJECTIONS}
    cfg = TorqueConfig(bit_width=bit_width, head_dim=int(w["w_q"].shape[0]) if head_dim is None else head_dim,
                       num_layers=num_layers, kv_heads=kv_heads, fused_weights=True, rotation_seed=rotation_seed)
    art = build_torque_artifact(model_name=model_name or Path(input_path).stem, architecture=architecture,
                                source_format=source_format, config=cfg, key_codebook=key_codebook,
                                value_codebook=value_codebook, **w)
    art.save(output_dir, force=force)
    return art
