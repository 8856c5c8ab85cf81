"""KV-cache transport between the prefill and decode ranks.

Two layers:

1. The packet protocol of hexgen2/transport.py:13-100, kept wire-compatible: an int64 header
   length, the UTF-8 JSON header {"version": 1, "metadata": ..., "tensors": [{name, shape,
   dtype}, ...]}, then each non-empty tensor as its own message, in header order, over the
   process group (NCCL on GPUs, Gloo on CPUs). Same limits (1 MiB header, 8 GiB payload,
   1024 tensors, 8 dims), same ValueError cases, checked before anything is allocated.
   `send_packet(..., packed=True)` adds "layout": "packed" to the header and sends all payload
   bytes as ONE message (each tensor at a 16-byte aligned offset); the receiver returns views
   of that one buffer. The KV dict returned by Engine.prefill already lives in one buffer, so
   packing it costs no copy.

2. KVHandoff: the B200 path. The decode rank exposes its destination buffer through CUDA IPC
   once; the prefill rank's gather-pack kernel then writes the live rows of every layer
   straight into it over NVLink (one kernel, no staging copy, no per-layer messages). Only a
   few bytes of control (lengths, readiness) travel through the process group.
"""
from __future__ import annotations

import json
import math

import torch
import torch.distributed as dist

DTYPES = {str(dtype): dtype for dtype in (
    torch.float16, torch.bfloat16, torch.float32, torch.float64,
    torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8, torch.bool,
)}
MAX_HEADER = 1024 * 1024
MAX_PAYLOAD = 8 * 1024 ** 3
MAX_TENSORS = 1024
MAX_DIMS = 8
ALIGN = 16


def wire_device():
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _elem_size(dtype_name: str) -> int:
    return torch.empty((), dtype=DTYPES[dtype_name]).element_size()


def validate_header(header) -> int:
    """Checks a packet header before any allocation; returns the payload size in bytes."""
    if header.get("version") != 1 or not isinstance(header.get("tensors"), list):
        raise ValueError("Unsupported tensor packet")
    items = header["tensors"]
    if len(items) > MAX_TENSORS:
        raise ValueError("Too many tensors")
    seen, total = set(), 0
    for item in items:
        name, shape, dtype = item.get("name"), item.get("shape"), item.get("dtype")
        if not isinstance(name, str) or name in seen or dtype not in DTYPES:
            raise ValueError("Invalid tensor name or dtype")
        if (not isinstance(shape, list) or len(shape) > MAX_DIMS
                or any(type(n) is not int or n < 0 for n in shape)):
            raise ValueError("Invalid tensor shape")
        total += math.prod(shape) * _elem_size(dtype)
        seen.add(name)
    if total > MAX_PAYLOAD:
        raise ValueError("Tensor packet exceeds memory limit")
    return total


def _packed_offsets(items):
    offs, o = [], 0
    for item in items:
        offs.append(o)
        o += math.prod(item["shape"]) * _elem_size(item["dtype"])
        o = (o + ALIGN - 1) // ALIGN * ALIGN
    return offs, o


def _send_bytes(buf: torch.Tensor, dst: int):
    if buf.numel():
        dist.send(buf, dst=dst)


def send_packet(tensors: dict, metadata, dst: int, packed: bool = False) -> int:
    """Sends a self-describing packet; returns the payload bytes (headers excluded)."""
    header = {"version": 1, "metadata": metadata, "tensors": [
        {"name": name, "shape": list(t.shape), "dtype": str(t.dtype)} for name, t in tensors.items()]}
    if packed:
        header["layout"] = "packed"
    payload = validate_header(header)
    encoded = json.dumps(header, allow_nan=False).encode("utf-8")
    if not 0 < len(encoded) <= MAX_HEADER:
        raise ValueError("Tensor metadata exceeds limit")
    device = wire_device()
    dist.send(torch.tensor([len(encoded)], dtype=torch.int64, device=device), dst=dst)
    dist.send(torch.frombuffer(bytearray(encoded), dtype=torch.uint8).to(device), dst=dst)
    if not packed:
        for t in tensors.values():
            t = t.detach().to(device).contiguous()
            if t.numel():
                dist.send(t, dst=dst)
        return payload
    offs, total = _packed_offsets(header["tensors"])
    region = _shared_region(list(tensors.values()), offs, total, device)
    if region is None:
        region = torch.zeros(total, dtype=torch.uint8, device=device)
        for t, o in zip(tensors.values(), offs):
            b = t.detach().to(device).contiguous().view(-1).view(torch.uint8)
            region[o:o + b.numel()].copy_(b)
    _send_bytes(region, dst)
    return payload


def _shared_region(ts, offs, total, device):
    """If the tensors already sit in one buffer at exactly the packed offsets (e.g. the KV dict
    from Engine.prefill), returns that byte range without copying."""
    if not ts or any(t.device != device or not t.is_contiguous() for t in ts):
        return None
    base = ts[0].data_ptr() - offs[0]
    if any(t.data_ptr() != base + o for t, o in zip(ts, offs)):
        return None
    storage = ts[0].untyped_storage()
    start = base - storage.data_ptr()
    if start < 0 or start + total > storage.nbytes():
        return None
    return torch.empty(0, dtype=torch.uint8, device=device).set_(storage, start, (total,))


def recv_packet(src: int):
    """Receives one packet; returns (tensors, metadata). Tensors are freshly allocated (per
    tensor, or views of one buffer for packed packets)."""
    device = wire_device()
    length = torch.empty(1, dtype=torch.int64, device=device)
    dist.recv(length, src=src)
    size = int(length.item())
    if not 0 < size <= MAX_HEADER:
        raise ValueError("Invalid tensor header length")
    encoded = torch.empty(size, dtype=torch.uint8, device=device)
    dist.recv(encoded, src=src)
    header = json.loads(bytes(encoded.cpu().tolist()).decode("utf-8"))
    validate_header(header)
    tensors = {}
    if header.get("layout") == "packed":
        offs, total = _packed_offsets(header["tensors"])
        region = torch.empty(total, dtype=torch.uint8, device=device)
        _send_or_recv = dist.recv
        if total:
            _send_or_recv(region, src=src)
        for item, o in zip(header["tensors"], offs):
            dt = DTYPES[item["dtype"]]
            n = math.prod(item["shape"]) * _elem_size(item["dtype"])
            tensors[item["name"]] = region[o:o + n].view(dt).view(item["shape"])
        return tensors, header["metadata"]
    for item in header["tensors"]:
        t = torch.empty(item["shape"], dtype=DTYPES[item["dtype"]], device=device)
        if t.numel():
            dist.recv(t, src=src)
        tensors[item["name"]] = t
    return tensors, header["metadata"]


def send_data(single_tensor, tensor_dict, dst, packed: bool = False):
    """Compatibility API (hexgen2/transport.py:83-89): token + {layer: kv}."""
    keys = list(tensor_dict)
    if any(type(k) is not int for k in keys):
        raise ValueError("KV-cache layer keys must be integers")
    return send_packet({"token": single_tensor, **{f"kv/{k}": tensor_dict[k] for k in keys}},
                       {"layers": keys}, dst, packed=packed)


def recv_data(src, num_layers=None, tensor_shape=None):
    """Compatibility API (hexgen2/transport.py:92-100)."""
    tensors, metadata = recv_packet(src)
    cache = {k: tensors[f"kv/{k}"] for k in metadata["layers"]}
    if num_layers is not None and len(cache) != num_layers:
        raise ValueError("Received KV-cache layer count differs from expected count")
    if tensor_shape is not None and any(tuple(t.shape) != tuple(tensor_shape) for t in cache.values()):
        raise ValueError("Received KV-cache shape differs from expected shape")
    return tensors["token"], cache


# ------------------------------------------------------------------------------------------
# NVLink direct handoff
# ------------------------------------------------------------------------------------------
class KVHandoff:
    """Direct prefill -> decode KV handoff over NVLink between two CUDA ranks.

    The receiver owns a destination buffer and shares it once through CUDA IPC (`expose`);
    the sender maps it (`attach`). From then on the sender's gather-pack kernel is given the
    mapped peer address as its destination, so the live rows of all layers cross NVLink inside
    one kernel with no staging copy and no per-layer messages. The control message (an int64
    tensor) is sent through the process group only after the kernel has completed, so the
    receiver never reads a partially written buffer.
    """

    def __init__(self, peer: int, group=None):
        from . import _lib
        self._lib = _lib
        self.peer, self.group = peer, group
        self.remote_ptr = None
        self._mapped = None
        self.local = None

    def _wire(self, t):
        return t.cuda() if dist.get_backend(self.group) == "nccl" else t

    # -------------------------------------------------------------- receiver side
    def expose(self, nbytes: int) -> torch.Tensor:
        """Allocates the receive buffer and sends (IPC handle, offset) to the peer."""
        import ctypes
        lib = self._lib.lib()
        self.local = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
        base, size = ctypes.c_void_p(), ctypes.c_size_t()
        self._lib.check(lib.hx_mem_range(self.local.data_ptr(), ctypes.byref(base), ctypes.byref(size)),
                        "hx_mem_range")
        handle = (ctypes.c_uint8 * 64)()
        self._lib.check(lib.hx_ipc_get_handle(base.value, handle), "hx_ipc_get_handle")
        offset = self.local.data_ptr() - base.value
        msg = torch.tensor(list(bytes(handle)) + list(offset.to_bytes(8, "little")), dtype=torch.uint8)
        dist.send(self._wire(msg), dst=self.peer, group=self.group)
        return self.local

    # -------------------------------------------------------------- sender side
    def attach(self) -> int:
        """Receives the peer's IPC handle and maps its buffer; returns the device address."""
        import ctypes
        msg = self._wire(torch.empty(72, dtype=torch.uint8))
        dist.recv(msg, src=self.peer, group=self.group)
        raw = bytes(msg.cpu().tolist())
        handle = (ctypes.c_uint8 * 64).from_buffer_copy(raw[:64])
        ptr = ctypes.c_void_p()
        self._lib.check(self._lib.lib().hx_ipc_open_handle(handle, ctypes.byref(ptr)),
                        "hx_ipc_open_handle")
        self._mapped = ptr.value
        self.remote_ptr = ptr.value + int.from_bytes(raw[64:72], "little")
        return self.remote_ptr

    def notify(self, nbytes: int, seq: int):
        """Sender: after the pack kernel finished, tell the receiver the bytes are in place."""
        torch.cuda.current_stream().synchronize()
        dist.send(self._wire(torch.tensor([nbytes, seq], dtype=torch.int64)), dst=self.peer,
                  group=self.group)

    def wait(self):
        """Receiver: blocks until the sender's notify; returns (nbytes, seq)."""
        msg = self._wire(torch.empty(2, dtype=torch.int64))
        dist.recv(msg, src=self.peer, group=self.group)
        n, seq = msg.cpu().tolist()
        return int(n), int(seq)

    def close(self):
        if self._mapped:
            self._lib.lib().hx_ipc_close_handle(self._mapped)
            self._mapped = None
