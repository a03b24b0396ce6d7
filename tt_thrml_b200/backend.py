"""The CUDA device backend: the object passed where the reference passes `ttnn`.

It offers the device calls the reference makes on ttnn (open_device,
close_device, open_mesh_device, close_mesh_device, synchronize_device,
MeshShape; tt_thrml/core.py:178-228, tt_thrml/mesh.py:25-26) on top of
torch's CUDA runtime.  Devices opened here are owned by the caller; executors
borrow them and never close them.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from types import SimpleNamespace


@dataclass
class CudaDevice:
    """One CUDA device plus the stream the executors launch on."""

    device_id: int
    _stream: object = field(default=None, repr=False)
    closed: bool = False

    @property
    def torch_device(self):
        import torch

        return torch.device("cuda", self.device_id)

    @property
    def stream(self):
        import torch

        if self._stream is None:
            self._stream = torch.cuda.Stream(device=self.torch_device)
        return self._stream

    def get_device_ids(self) -> list[int]:
        return [self.device_id]


@dataclass
class CudaMeshDevice:
    """A set of CUDA devices driven together (the MeshDevice counterpart)."""

    mesh_shape: tuple[int, ...]
    devices: list[CudaDevice]
    closed: bool = False

    def get_device_ids(self) -> list[int]:
        return [d.device_id for d in self.devices]


def _require_cuda():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available: the B200 backend has no CPU fallback")
    return torch


class _CudaBackend:
    @staticmethod
    def MeshShape(*dims):
        return SimpleNamespace(dims=tuple(int(d) for d in dims))

    def open_device(self, *, device_id: int = 0) -> CudaDevice:
        torch = _require_cuda()
        if not 0 <= int(device_id) < torch.cuda.device_count():
            raise ValueError(f"CUDA device {device_id} does not exist ({torch.cuda.device_count()} visible)")
        torch.cuda.init()
        return CudaDevice(int(device_id))

    def close_device(self, device) -> None:
        import torch

        if isinstance(device, CudaDevice) and not device.closed:
            with torch.cuda.device(device.device_id):
                torch.cuda.synchronize()
            device.closed = True

    def open_mesh_device(self, *, mesh_shape, physical_device_ids=None, num_command_queues: int = 1, offset=None):
        torch = _require_cuda()
        dims = tuple(getattr(mesh_shape, "dims", mesh_shape))
        n = 1
        for d in dims:
            n *= int(d)
        ids = list(physical_device_ids) if physical_device_ids is not None else list(range(n))
        if len(ids) != n:
            raise ValueError(f"mesh {dims} needs {n} device ids, got {len(ids)}")
        if any(not 0 <= i < torch.cuda.device_count() for i in ids):
            raise ValueError(f"mesh device ids {ids} exceed the {torch.cuda.device_count()} visible devices")
        return CudaMeshDevice(dims, [CudaDevice(int(i)) for i in ids])

    def close_mesh_device(self, device) -> None:
        for d in getattr(device, "devices", []):
            self.close_device(d)
        device.closed = True

    def synchronize_device(self, device) -> None:
        import torch

        for d in getattr(device, "devices", [device]):
            with torch.cuda.device(d.device_id):
                torch.cuda.synchronize()


cuda = _CudaBackend()
