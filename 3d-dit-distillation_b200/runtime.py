"""Plugin contract of the lat_dit track, mirrored for the drop-in boundary.

Same names, fields and behaviour as the reference's
``BK/kandi3d_image23d/runtime.py`` (``FlowMatchSamplingParams`` ``:31-63``,
``LatDitConditioning`` ``:100-117``, ``resolve`` ``:209-215``) and
``BK/kandi3d_image23d/lat_dit_protocol.py`` (``LatDitGenerator`` ``:39-151``).
When the reference package ``kandi3d_image23d`` is importable, its classes
are used instead so a ``Solution`` built here is a real subclass of the
harness's ``LatDitGenerator``.
"""
from __future__ import annotations

import time
from abc import ABC, abstractmethod
from dataclasses import asdict, dataclass, is_dataclass
from typing import Any, Dict, Optional, Tuple, TypeVar, Union

import torch

T = TypeVar("T", bound="RuntimeParams")


@dataclass(frozen=True)
class RuntimeParams:
    """None-aware merge: default <- other <- kwargs."""

    def merge(self: T, other: Optional[T] = None, **kwargs: Any) -> T:
        base = asdict(self)
        if other is not None:
            for k, v in asdict(other).items():
                if v is not None:
                    base[k] = v
        for k, v in kwargs.items():
            if v is not None and k in base:
                base[k] = tuple(float(x) for x in v) if k == "cfg_range" and isinstance(v, (list, tuple)) else v
        return type(self)(**base)


@dataclass(frozen=True)
class FlowMatchSamplingParams(RuntimeParams):
    guidance_scale: float = 2.5
    cfg_range: Tuple[float, float] = (0.5, 1.0)
    rescale_t: float = 3.0
    num_inference_steps: int = 50

    @classmethod
    def from_yaml_section(cls, section: Dict[str, Any]) -> "FlowMatchSamplingParams":
        cr = section.get("cfg_range", [0.5, 1.0])
        cr = tuple(float(x) for x in cr) if isinstance(cr, (list, tuple)) else (0.5, 1.0)
        return cls(guidance_scale=float(section.get("cfg", section.get("guidance_scale", 2.5))), cfg_range=cr,
                   rescale_t=float(section.get("rescale_t", 3.0)),
                   num_inference_steps=int(section.get("num_inference_steps", 50)))

    @classmethod
    def from_dict(cls, data: Optional[Dict[str, Any]]) -> "FlowMatchSamplingParams":
        if not data:
            return cls()
        cr = data.get("cfg_range", (0.5, 1.0))
        return cls(guidance_scale=float(data.get("guidance_scale", 2.5)), cfg_range=tuple(cr),
                   rescale_t=float(data.get("rescale_t", 3.0)),
                   num_inference_steps=int(data.get("num_inference_steps", 50)))


@dataclass(frozen=True)
class LatDitConditioning:
    """DINOv3 conditioning bundle: dino_features [B, 4101, 1280]."""
    dino_features: "torch.Tensor"
    dino_token: Optional["torch.Tensor"] = None
    batch_size: int = 1
    nfaces: Optional["torch.Tensor"] = None

    def to_data_dict(self) -> Dict[str, Any]:
        dd: Dict[str, Any] = {"dino_features": self.dino_features, "batch_size": self.batch_size}
        if self.dino_token is not None:
            dd["dino_token"] = self.dino_token
        if self.nfaces is not None:
            dd["nfaces"] = self.nfaces
        return dd


def resolve(default: T, override: Optional[T] = None, **kwargs: Any) -> T:
    return default.merge(override, **kwargs)


_OMIT = object()


def _json_safe(value: Any) -> Any:
    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    if is_dataclass(value):
        return _json_safe(asdict(value))
    if isinstance(value, dict):
        out = {}
        for k, v in value.items():
            c = _json_safe(v)
            if c is not _OMIT:
                out[str(k)] = c
        return out
    if isinstance(value, (list, tuple)):
        return [c for c in (_json_safe(v) for v in value) if c is not _OMIT]
    return _OMIT


class LatDitGenerator(ABC):
    """Participant contract: implement ``from_pretrained`` and ``generate_impl``;
    ``generate`` is final (it syncs CUDA, times the call and records
    ``last_run_metadata``)."""

    last_run_metadata: Dict[str, Any]

    def __init_subclass__(cls, **kwargs: Any) -> None:
        super().__init_subclass__(**kwargs)
        if "generate" in cls.__dict__:
            raise TypeError(f"{cls.__name__} must not override LatDitGenerator.generate(); implement generate_impl()")

    @classmethod
    @abstractmethod
    def from_pretrained(cls, pretrained_model_name_or_path: str,
                        device: Optional[Union[torch.device, str, int]] = None,
                        torch_dtype: Optional[torch.dtype] = None, **kwargs) -> "LatDitGenerator":
        raise NotImplementedError

    def generate(self, vox_idxs: list, *, conditioning: LatDitConditioning,
                 sampling: Optional[FlowMatchSamplingParams] = None, generator: Optional[torch.Generator] = None,
                 **sampling_kwargs) -> list:
        resolved = sampling or getattr(self, "_default_runtime", FlowMatchSamplingParams())
        metadata: Dict[str, Any] = {
            "generator_class": f"{type(self).__module__}.{type(self).__qualname__}",
            "inputs": {
                "sampling": _json_safe(resolved),
                "sampling_kwargs": _json_safe(sampling_kwargs),
                "batch_size": int(conditioning.batch_size),
                "num_voxels": [int(v.shape[0]) for v in vox_idxs],
                "generator_seed": int(generator.initial_seed()) if generator is not None else None,
            },
        }
        dev = next((v.device for v in vox_idxs if torch.is_tensor(v) and v.is_cuda), None)
        if dev is not None:
            torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        try:
            out = self.generate_impl(vox_idxs, conditioning=conditioning, sampling=sampling, generator=generator,
                                     **sampling_kwargs)
            if dev is not None:
                torch.cuda.synchronize(dev)
            metadata["elapsed_seconds"] = float(time.perf_counter() - t0)
            metadata["status"] = "ok"
            self.last_run_metadata = metadata
            return out
        except Exception as exc:
            if dev is not None:
                torch.cuda.synchronize(dev)
            metadata["elapsed_seconds"] = float(time.perf_counter() - t0)
            metadata["status"] = "error"
            metadata["error_type"] = type(exc).__name__
            self.last_run_metadata = metadata
            raise

    @abstractmethod
    def generate_impl(self, vox_idxs: list, *, conditioning: LatDitConditioning,
                      sampling: Optional[FlowMatchSamplingParams] = None,
                      generator: Optional[torch.Generator] = None, **sampling_kwargs: Any) -> list:
        raise NotImplementedError


try:  # use the harness's own classes when the reference package is on the path
    from kandi3d_image23d.lat_dit_protocol import LatDitGenerator as _RefGenerator  # type: ignore
    from kandi3d_image23d.runtime import (FlowMatchSamplingParams as _RefParams,  # type: ignore
                                          LatDitConditioning as _RefCond, resolve as _ref_resolve)
    LatDitGenerator = _RefGenerator  # noqa: F811
    FlowMatchSamplingParams = _RefParams  # noqa: F811
    LatDitConditioning = _RefCond  # noqa: F811
    resolve = _ref_resolve  # noqa: F811
except Exception:  # the mirror above is the contract
    pass
