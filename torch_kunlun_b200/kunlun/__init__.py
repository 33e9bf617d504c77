"""The ``torch.kunlun`` device module.

Same surface as the reference's torch_kunlun/kunlun/__init__.py:16-279:
device queries, synchronisation, memory statistics, the cluster-budget calls,
pinned-memory queries, ``Stream`` (a real ``torch.Stream`` subclass), ``Event``,
``current_stream`` / ``default_stream`` / ``set_stream`` and the ``stream()``
context manager.  Underneath, a kunlun device is a CUDA device of this
machine, streams are CUDA streams and events are CUDA events, so
``Event.query()`` does not block and ``Event.elapsed_time()`` works (the
reference raises for the latter, torch_kunlun/kunlun/__init__.py:219-220).
"""

from __future__ import annotations

from collections import namedtuple
from typing import List, Optional, Tuple

import torch

from .. import _C

DeviceProperties = namedtuple(
    "DeviceProperties",
    ["name", "total_memory", "multi_processor_count", "warp_size", "major", "minor", "model"],
)


def is_available() -> bool:
    return device_count() > 0


def device_count() -> int:
    return int(_C.device_count())


def current_device() -> int:
    return int(_C.current_device())


def set_device(device) -> None:
    _C.set_device(_device_index(device))


def synchronize(device: Optional[int] = None) -> None:
    if device is not None:
        set_device(device)
    _C.synchronize()


def get_device_properties(device=None) -> DeviceProperties:
    return DeviceProperties(**_C.get_device_properties(_device_index(device)))


def get_device_name(device=None) -> str:
    return get_device_properties(device).name


def get_device_capability(device=None) -> Tuple[int, int]:
    props = get_device_properties(device)
    return props.major, props.minor


def memory_allocated(device: Optional[int] = None) -> int:
    return int(_C.memory_allocated(-1 if device is None else _device_index(device)))


def max_memory_allocated(device: Optional[int] = None) -> int:
    return int(_C.max_memory_allocated(-1 if device is None else _device_index(device)))


def reset_peak_memory_stats(device: Optional[int] = None) -> None:
    _C.reset_peak_memory_stats(-1 if device is None else _device_index(device))


def memory_reserved(device: Optional[int] = None) -> int:
    return int(_C.memory_reserved(-1 if device is None else _device_index(device)))


def empty_cache() -> None:
    _C.empty_cache()


def xdnn_version() -> str:
    """Kept for API compatibility; there is no XDNN library on B200."""
    return str(_C.xdnn_version())


def cluster_budget() -> int:
    return int(_C.cluster_budget())


def sdnn_budget() -> int:
    return int(_C.sdnn_budget())


def set_cluster_budget(nclusters: int, nsdnn: Optional[int] = None) -> int:
    """Kept for API compatibility (K200 cluster partitioning has no B200
    counterpart): the values are validated and reported back, kernels always
    use the whole GPU."""
    nsdnn = nclusters if nsdnn is None else nsdnn
    return int(_C.set_cluster_budget(int(nclusters), int(nsdnn)))


def is_pinned_ptr(address: int) -> bool:
    """True if ``address`` is page-locked host memory (CUDA host allocation)."""
    return bool(_C.is_pinned_ptr(int(address)))


def is_pinned_tensor(tensor: torch.Tensor) -> bool:
    if tensor.device.type != "cpu":
        return False
    return is_pinned_ptr(tensor.data_ptr())


def _is_in_bad_fork() -> bool:
    return False


def manual_seed_all(seed: int) -> None:
    # Random number generation on the device is not part of this backend.
    return None


def get_amp_supported_dtype() -> List[torch.dtype]:
    return [torch.float16]


def _device_index(device) -> int:
    if device is None:
        return current_device()
    if isinstance(device, str):
        device = torch.device(device)
    if isinstance(device, torch.device):
        if device.type not in ("kunlun", "privateuseone"):
            raise ValueError(f"expected a kunlun device, got {device}")
        return current_device() if device.index is None else int(device.index)
    return int(device)


_PRIVATEUSE1_DEVICE_TYPE = int(torch._C._autograd.DeviceType.PrivateUse1.value)
# (device, stream id) -> id() of the one Stream object that owns (and will
# destroy) the stream; wrappers of the same stream made by current_stream()
# and friends do not own it.
_OWNED_STREAMS = {}


class Stream(torch.Stream):
    """A kunlun stream that is also a real ``torch.Stream``.

    Without ``stream_id`` a new stream is created and owned; with it the
    object wraps an existing one (``0`` is the device's default stream).
    """

    def __new__(cls, device=None, stream_id=None, priority: int = 0):
        index = _device_index(device)
        owned = stream_id is None
        raw_id = int(_C.create_stream(index, int(priority))) if owned else int(stream_id)
        obj = super().__new__(cls, raw_id, index, _PRIVATEUSE1_DEVICE_TYPE)
        if owned:
            _OWNED_STREAMS[(index, raw_id)] = id(obj)
        return obj

    def __init__(self, device=None, stream_id=None, priority: int = 0):
        pass

    @property
    def _index(self) -> int:
        return int(self.device_index)

    def wait_event(self, event: "Event") -> None:
        _C.stream_wait_event(self._index, self.stream_id, event.event_id)

    def wait_stream(self, other: "Stream") -> None:
        event = Event()
        event.record(other)
        event.wait(self)

    def record_event(self, event: Optional["Event"] = None) -> "Event":
        event = Event() if event is None else event
        event.record(self)
        return event

    def query(self) -> bool:
        return bool(_C.stream_query(self._index, self.stream_id))

    def synchronize(self) -> None:
        _C.synchronize_stream(self._index, self.stream_id)

    def __del__(self):
        try:
            key = (int(self.device_index), int(self.stream_id))
            if _OWNED_STREAMS.get(key) == id(self):
                del _OWNED_STREAMS[key]
                _C.destroy_stream(*key)
        except Exception:
            pass


class Event:
    """A kunlun event (a CUDA event on the kunlun device)."""

    def __init__(self, enable_timing: bool = False, device=None):
        self.enable_timing = enable_timing
        self._device = _device_index(device)
        self.event_id = int(_C.event_create(self._device, bool(enable_timing)))

    def record(self, stream: Optional[Stream] = None) -> None:
        target = stream if stream is not None else current_stream(self._device)
        _C.event_record(self.event_id, int(target.device_index), target.stream_id)

    def wait(self, stream: Optional[Stream] = None) -> None:
        target = stream if stream is not None else current_stream(self._device)
        _C.stream_wait_event(int(target.device_index), target.stream_id, self.event_id)

    def query(self) -> bool:
        return bool(_C.event_query(self.event_id))

    def synchronize(self) -> None:
        _C.event_synchronize(self.event_id)

    def elapsed_time(self, other: "Event") -> float:
        return float(_C.event_elapsed_time(self.event_id, other.event_id))

    def __del__(self):
        if getattr(self, "event_id", None):
            try:
                _C.event_destroy(self.event_id)
            except Exception:
                pass


def current_stream(device=None) -> Stream:
    index = _device_index(device)
    return Stream(index, stream_id=int(_C.current_stream(index)))


def default_stream(device=None) -> Stream:
    index = _device_index(device)
    return Stream(index, stream_id=int(_C.default_stream(index)))


def set_stream(stream: Stream) -> None:
    _C.set_stream(int(stream.device_index), stream.stream_id)


class _StreamContext:
    def __init__(self, stream: Stream):
        self.stream = stream
        self.prev = None

    def __enter__(self):
        self.prev = current_stream(int(self.stream.device_index))
        set_stream(self.stream)
        return self.stream

    def __exit__(self, exc_type, exc_value, traceback):
        if self.prev is not None:
            set_stream(self.prev)
        return False


def stream(stream_obj: Stream) -> _StreamContext:
    return _StreamContext(stream_obj)


from .attention import scaled_dot_product_attention  # noqa: E402

__all__ = [
    "Stream",
    "Event",
    "scaled_dot_product_attention",
    "is_available",
    "device_count",
    "current_device",
    "set_device",
    "synchronize",
    "current_stream",
    "default_stream",
    "set_stream",
    "stream",
]
