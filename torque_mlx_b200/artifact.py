"""Torque artifacts: fused attention weights plus the runtime profile.

Same on-disk format as the reference (src/torque_mlx/artifact.py; contract
docs/contracts/model-artifact.md): a directory with ``manifest.json``
(format ``torque-mlx-artifact`` v1, runtime config, K/V codebooks, weight
names, metadata) and ``weights.npz`` (``w_q, w_k, w_v, w_o`` already fused
with Pi).  Artifacts written by either project load in the other, and
``build_cache()`` returns this project's GPU cache with the artifact's exact
codebooks and rotation (artifact.py:157-162).
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field, replace
from pathlib import Path
from typing import Any, Mapping

import numpy as np

from .cache import TorqueKVCache
from .config import RotationMode, TorqueConfig
from .conversion import FusedAttentionWeights, fuse_attention_weights
from .quantization import Codebook, build_gaussian_codebook
from .rotation import RotationSpec

ARTIFACT_FORMAT = "torque-mlx-artifact"
ARTIFACT_VERSION = 1
DEFAULT_WEIGHTS_FILE = "weights.npz"
DEFAULT_MANIFEST_FILE = "manifest.json"
_DEFAULT_WEIGHT_NAMES = {"w_q": "w_q", "w_k": "w_k", "w_v": "w_v", "w_o": "w_o"}


def _plain(value: Any) -> Any:
    """JSON-serialisable copy (numpy scalars -> Python scalars)."""
    if isinstance(value, dict):
        return {str(k): _plain(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_plain(v) for v in value]
    if isinstance(value, np.generic):
        return value.item()
    return value


@dataclass(frozen=True, slots=True)
class TorqueArtifactManifest:
    """Manifest fields and checks of artifact.py:40-137."""

    model_name: str
    architecture: str
    source_format: str
    runtime_config: TorqueConfig
    key_codebook: Codebook
    value_codebook: Codebook
    weights_file: str = DEFAULT_WEIGHTS_FILE
    format_name: str = ARTIFACT_FORMAT
    format_version: int = ARTIFACT_VERSION
    weight_names: dict[str, str] = field(default_factory=lambda: dict(_DEFAULT_WEIGHT_NAMES))
    extra_metadata: dict[str, object] = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.runtime_config.validate()
        if not self.runtime_config.fused_weights:
            raise ValueError("Artifact runtime_config must enable fused_weights")
        if self.format_name != ARTIFACT_FORMAT:
            raise ValueError(f"Unsupported artifact format: {self.format_name}")
        if self.format_version != ARTIFACT_VERSION:
            raise ValueError(f"Unsupported artifact version: {self.format_version}")

    @classmethod
    def from_dict(cls, payload: Mapping[str, object]) -> "TorqueArtifactManifest":
        required = ("model_name", "architecture", "source_format", "runtime_config", "key_codebook",
                    "value_codebook")
        missing = [k for k in required if k not in payload]
        if missing:
            raise ValueError(f"Missing required fields: {', '.join(missing)}")
        rc = payload["runtime_config"]
        if not isinstance(rc, Mapping):
            raise ValueError("runtime_config must be an object")
        config = TorqueConfig(bit_width=int(rc["bit_width"]), head_dim=int(rc["head_dim"]),
                              num_layers=int(rc["num_layers"]), kv_heads=int(rc["kv_heads"]),
                              fused_weights=bool(rc["fused_weights"]),
                              rotation_mode=RotationMode(str(rc["rotation_mode"])),
                              rotation_seed=int(rc["rotation_seed"]))
        names = dict(payload.get("weight_names", {})) or dict(_DEFAULT_WEIGHT_NAMES)
        return cls(model_name=str(payload["model_name"]), architecture=str(payload["architecture"]),
                   source_format=str(payload["source_format"]), runtime_config=config,
                   key_codebook=Codebook.from_dict(dict(payload["key_codebook"])),
                   value_codebook=Codebook.from_dict(dict(payload["value_codebook"])),
                   weights_file=str(payload.get("weights_file", DEFAULT_WEIGHTS_FILE)),
                   format_name=str(payload.get("format_name", ARTIFACT_FORMAT)),
                   format_version=int(payload.get("format_version", ARTIFACT_VERSION)),
                   weight_names={str(k): str(v) for k, v in names.items()},
                   extra_metadata={str(k): _plain(v) for k, v in dict(payload.get("extra_metadata", {})).items()})

    def to_dict(self) -> dict[str, object]:
        rc = self.runtime_config
        return {
            "format_name": self.format_name, "format_version": self.format_version,
            "model_name": self.model_name, "architecture": self.architecture,
            "source_format": self.source_format, "variant_id": rc.variant_id,
            "runtime_config": {"bit_width": rc.bit_width, "head_dim": rc.head_dim, "num_layers": rc.num_layers,
                               "kv_heads": rc.kv_heads, "fused_weights": rc.fused_weights,
                               "rotation_mode": rc.rotation_mode.value, "rotation_seed": rc.rotation_seed},
            "weights_file": self.weights_file, "weight_names": dict(self.weight_names),
            "key_codebook": self.key_codebook.to_dict(), "value_codebook": self.value_codebook.to_dict(),
            "extra_metadata": _plain(self.extra_metadata),
        }


@dataclass(frozen=True, slots=True)
class TorqueArtifact:
    manifest: TorqueArtifactManifest
    fused_weights: FusedAttentionWeights

    @property
    def runtime_config(self) -> TorqueConfig:
        return self.manifest.runtime_config

    @property
    def key_codebook(self) -> Codebook:
        return self.manifest.key_codebook

    @property
    def value_codebook(self) -> Codebook:
        return self.manifest.value_codebook

    def build_cache(self, **cache_kwargs) -> TorqueKVCache:
        """The drop-in hook: a GPU packed cache with this artifact's config and
        codebooks (extra keyword arguments go to TorqueKVCache)."""
        return TorqueKVCache(config=self.runtime_config, key_codebook=self.key_codebook,
                             value_codebook=self.value_codebook, **cache_kwargs)

    def save(self, directory: str | Path, *, force: bool = False) -> Path:
        target = Path(directory)
        if target.exists() and any(target.iterdir()) and not force:
            raise FileExistsError(
                f"Refusing to overwrite non-empty artifact directory {target}; pass force=True to replace it")
        target.mkdir(parents=True, exist_ok=True)
        (target / DEFAULT_MANIFEST_FILE).write_text(json.dumps(self.manifest.to_dict(), indent=2, sort_keys=True),
                                                    encoding="utf-8")
        fw, names = self.fused_weights, self.manifest.weight_names
        np.savez_compressed(target / self.manifest.weights_file,
                            **{names["w_q"]: fw.w_q, names["w_k"]: fw.w_k, names["w_v"]: fw.w_v,
                               names["w_o"]: fw.w_o})
        return target

    def summary(self) -> dict[str, object]:
        rc, fw = self.runtime_config, self.fused_weights
        return {
            "format_name": self.manifest.format_name, "format_version": self.manifest.format_version,
            "model_name": self.manifest.model_name, "architecture": self.manifest.architecture,
            "source_format": self.manifest.source_format, "variant_id": rc.variant_id,
            "weights_file": self.manifest.weights_file,
            "runtime_config": self.manifest.to_dict()["runtime_config"],
            "weight_shapes": {k: list(getattr(fw, k).shape) for k in ("w_q", "w_k", "w_v", "w_o")},
            "key_codebook": {"name": self.key_codebook.name, "bit_width": self.key_codebook.bit_width,
                             "centroid_count": int(self.key_codebook.centroids.size)},
            "value_codebook": {"name": self.value_codebook.name, "bit_width": self.value_codebook.bit_width,
                               "centroid_count": int(self.value_codebook.centroids.size)},
            "extra_metadata": _plain(self.manifest.extra_metadata),
        }

    @classmethod
    def load(cls, directory: str | Path) -> "TorqueArtifact":
        target = Path(directory)
        mpath = target / DEFAULT_MANIFEST_FILE
        if not mpath.exists():
            raise FileNotFoundError(f"Artifact manifest not found: {mpath}")
        manifest = TorqueArtifactManifest.from_dict(json.loads(mpath.read_text(encoding="utf-8")))
        wpath = target / manifest.weights_file
        if not wpath.exists():
            raise FileNotFoundError(f"Artifact weights not found: {wpath}")
        with np.load(wpath) as data:
            ws = {k: np.asarray(data[manifest.weight_names[k]], dtype=np.float32) for k in ("w_q", "w_k", "w_v", "w_o")}
        return cls(manifest=manifest,
                   fused_weights=FusedAttentionWeights(**ws, rotation_seed=manifest.runtime_config.rotation_seed))


def build_torque_artifact(*, model_name: str, architecture: str, source_format: str, config: TorqueConfig,
                          w_q, w_k, w_v, w_o, rotation: RotationSpec | None = None,
                          key_codebook: Codebook | None = None, value_codebook: Codebook | None = None,
                          extra_metadata: Mapping[str, object] | None = None) -> TorqueArtifact:
    """Fuse the weights and assemble an artifact (artifact.py:246-296): the
    runtime config is forced to fused_weights, codebooks default to the
    seeded Gaussian ones (K: rotation_seed, V: rotation_seed + 1)."""
    rc = replace(config, fused_weights=True)
    rotation = rotation or RotationSpec.from_seed(head_dim=rc.head_dim, seed=rc.rotation_seed)
    key_codebook = key_codebook or build_gaussian_codebook(rc.bit_width, seed=rc.rotation_seed)
    value_codebook = value_codebook or build_gaussian_codebook(rc.bit_width, seed=rc.rotation_seed + 1)
    fused = fuse_attention_weights(w_q=w_q, w_k=w_k, w_v=w_v, w_o=w_o, rotation=rotation)
    meta: dict[str, object] = {"input_dim": int(np.shape(w_q)[1]), "output_dim": int(np.shape(w_o)[0])}
    if extra_metadata:
        meta.update({str(k): _plain(v) for k, v in extra_metadata.items()})
    manifest = TorqueArtifactManifest(model_name=model_name, architecture=architecture, source_format=source_format,
                                      runtime_config=rc, key_codebook=key_codebook, value_codebook=value_codebook,
                                      extra_metadata=meta)
    return TorqueArtifact(manifest=manifest, fused_weights=fused)


def convert_npz_checkpoint(*, input_path: str | Path, output_dir: str | Path, model_name: str | None,
                           architecture: str, source_format: str, bit_width: int, num_layers: int, kv_heads: int,
                           rotation_seed: int, head_dim: int | None = None, key_codebook: Codebook | None = None,
                           value_codebook: Codebook | None = None, force: bool = False) -> TorqueArtifact:
    """NPZ (w_q, w_k, w_v, w_o) -> saved artifact (artifact.py:299-343)."""
    with np.load(input_path) as ck:
        if any(k not in ck for k in ("w_q", "w_k", "w_v", "w_o")):
            raise ValueError("Expected NPZ checkpoint to contain w_q, w_k, w_v, and w_o arrays")
        ws = {k: np.asarray(ck[k]) for k in ("w_q", "w_k", "w_v", "w_o")}
    config = TorqueConfig(bit_width=bit_width, head_dim=int(ws["w_q"].shape[0]) if head_dim is None else head_dim,
                          num_layers=num_layers, kv_heads=kv_heads, fused_weights=True, rotation_seed=rotation_seed)
    art = build_torque_artifact(model_name=model_name or Path(input_path).stem, architecture=architecture,
                                source_format=source_format, config=config, key_codebook=key_codebook,
                                value_codebook=value_codebook, **ws)
    art.save(output_dir, force=force)
    return art


def load_torque_artifact(directory: str | Path) -> TorqueArtifact:
    return TorqueArtifact.load(directory)
