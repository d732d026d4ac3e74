"""Device array intake: a bound plane's address, shape, dtype and device.

The reference binds host planes through the buffer protocol
(hawk/runtime.py:401-423).  The b200 path binds DEVICE planes, from any object
that describes one:

* a ``torch.Tensor`` on a CUDA device,
* an object with ``__cuda_array_interface__`` (CuPy, Numba, ...),
* an object with ``__dlpack__`` (read through ``torch.from_dlpack``).

A host array is refused: the device path copies nothing and has no CPU
fallback.  Nothing here allocates.
"""

from __future__ import annotations

from dataclasses import dataclass

from .errors import HawkError

_TYPESTR = {"<f8": "float64", "<f4": "float32", "<i4": "int32", "<i8": "int64", "<u4": "uint32",
            "|b1": "bool", "<f2": "float16"}
_ITEMSIZE = {"float64": 8, "float32": 4, "int32": 4, "int64": 8, "uint32": 4, "bool": 1, "float16": 2}


@dataclass
class Plane:
    """One bound array as the launch sees it."""

    ptr: int
    shape: tuple
    strides: tuple          # in elements
    dtype: str
    device: int | None      # CUDA ordinal, None for host memory
    readonly: bool
    keep: object            # the owner, kept alive while bound

    @property
    def contiguous(self) -> bool:
        expect = 1
        for extent, stride in zip(reversed(self.shape), reversed(self.strides)):
            if extent > 1 and stride != expect:
                return False
            expect *= max(extent, 1)
        return True

    @property
    def size(self) -> int:
        n = 1
        for e in self.shape:
            n *= e
        return n


def _torch_dtype_name(dt) -> str:
    name = str(dt).replace("torch.", "")
    return {"double": "float64", "float": "float32", "int": "int32", "long": "int64"}.get(name, name)


def from_torch(t) -> Plane:
    device = t.device.index if t.device.type == "cuda" else None
    if t.device.type == "cuda" and device is None:
        import torch
        device = torch.cuda.current_device()
    return Plane(ptr=int(t.data_ptr()), shape=tuple(int(e) for e in t.shape),
                 strides=tuple(int(s) for s in t.stride()), dtype=_torch_dtype_name(t.dtype),
                 device=device, readonly=False, keep=t)


def from_cai(obj) -> Plane:
    cai = obj.__cuda_array_interface__
    ptr, readonly = cai["data"]
    dtype = _TYPESTR.get(cai["typestr"], cai["typestr"])
    shape = tuple(int(e) for e in cai["shape"])
    item = _ITEMSIZE.get(dtype, 1)
    if cai.get("strides") is None:
        strides, acc = [], 1
        for e in reversed(shape):
            strides.append(acc)
            acc *= e
        strides = tuple(reversed(strides))
    else:
        strides = tuple(int(s) // item for s in cai["strides"])
    device = None
    try:                                     # the pointer's device, through the CUDA runtime
        from cuda.bindings import runtime as cudart
        err, attrs = cudart.cudaPointerGetAttributes(ptr)
        if int(err) == 0 and int(attrs.type) in (2, 3):
            device = int(attrs.device)
    except Exception:                        # noqa: BLE001 -- no runtime: assume the current device
        device = 0
    return Plane(ptr=int(ptr or 0), shape=shape, strides=strides, dtype=dtype, device=device,
                 readonly=bool(readonly), keep=obj)


def as_plane(name: str, obj) -> Plane:
    """The plane of one bound array, or a refusal naming ``name``."""
    try:
        import torch
    except ImportError:                      # pragma: no cover - torch is in the image
        torch = None
    if torch is not None and isinstance(obj, torch.Tensor):
        return from_torch(obj)
    if hasattr(obj, "__cuda_array_interface__"):
        return from_cai(obj)
    if hasattr(obj, "__dlpack__") and torch is not None and not hasattr(obj, "__array_interface__"):
        return from_torch(torch.from_dlpack(obj))
    if hasattr(obj, "__array_interface__") or hasattr(obj, "__array__"):
        raise HawkError(f"argument {name!r}: a host array was bound, but the b200 path binds device "
                        "planes only (it copies nothing): pass a CUDA tensor, e.g. "
                        f"torch.as_tensor({name}, device='cuda')")
    raise HawkError(f"argument {name!r}: {type(obj).__name__} is not a device array "
                    "(no __cuda_array_interface__ or __dlpack__)")
