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
    receiver never reads a partially written buffer. Nothing here stops a second pack from
    overwriting bytes the receiver has not consumed yet: a sender that reuses the buffer waits
    for the receiver's release first (the serving loop reserves regions of a ring and frees
    them on the decode rank's release message, serving.ByteRing).
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


# ------------------------------------------------------------------------------------------
# KV re-sharding between groups of different tensor-parallel sizes
# ------------------------------------------------------------------------------------------
def reshard_plan(n_kv_heads: int, src_tp: int, dst_tp: int) -> list[tuple[int, int, int, int]]:
    """Slice moves that turn a cache sharded over src_tp ranks (rank i holds KV heads
    [i*h/src_tp, (i+1)*h/src_tp)) into one sharded over dst_tp ranks: a list of
    (src_rank, dst_rank, head_lo, head_hi) in global head indices, by destination rank then head.
    The reference concatenates all shards on the head dimension and would then split
    (hexgen/llama/tensor_parallel_dim_concat.py:9-21); these moves give the same per-rank caches
    without materialising the full one. Raises ValueError if a TP size does not divide the heads."""
    if src_tp <= 0 or dst_tp <= 0 or n_kv_heads % src_tp or n_kv_heads % dst_tp:
        raise ValueError(f"{n_kv_heads} KV heads cannot be split {src_tp} and {dst_tp} ways")
    hs, hd = n_kv_heads // src_tp, n_kv_heads // dst_tp
    plan = []
    for dst in range(dst_tp):
        lo, hi = dst * hd, (dst + 1) * hd
        for src in range(src_tp):
            a, b = max(lo, src * hs), min(hi, (src + 1) * hs)
            if a < b:
                plan.append((src, dst, a, b))
    return plan


def _cache_geometry(caches: dict):
    """(layer-0 view, layers, layer stride in bytes) of an engine's all-layer cache handed out
    as per-layer views {layer: [B, cap, 2, hkv, d]}."""
    n = len(caches)
    big0 = caches[0]
    stride = (caches[1].data_ptr() - big0.data_ptr()) if n > 1 else 0
    if any(caches[i].data_ptr() != big0.data_ptr() + i * stride for i in range(n)):
        raise ValueError("expected one all-layer cache (per-layer views at a fixed stride)")
    if big0.stride(-1) != 1 or big0.stride(-2) != big0.shape[-1]:
        raise ValueError("cache rows must be contiguous [2, hkv, d]")
    return big0, n, stride


def head_slice_bytes(caches: dict, lengths: list[int], n_heads: int) -> list[int]:
    """Packed bytes per request of a head slice (K slab then V slab, all layers)."""
    big0, n, _ = _cache_geometry(caches)
    return [2 * n * L * n_heads * big0.shape[-1] * big0.element_size() for L in lengths]


def pack_kv_heads(caches: dict, rows: list[int], lengths: list[int], head_lo: int, head_hi: int,
                  dst, dst_offsets: list[int]):
    """Gather-packs KV heads [head_lo, head_hi) (indices local to this cache) of the live rows
    of requests `rows` (batch rows of the all-layer cache) into `dst` (a CUDA tensor, or a peer
    address from KVHandoff.attach): per request, at dst_offsets[r], the K slab
    [layers][L][heads][d] followed by the V slab. Two gather-pack launches (K, V)."""
    from . import ops
    big0, n, lstride = _cache_geometry(caches)
    hk, d, elem = big0.shape[-2], big0.shape[-1], big0.element_size()
    if not 0 <= head_lo < head_hi <= hk:
        raise ValueError(f"head range [{head_lo}, {head_hi}) outside the cache's {hk} heads")
    nh = head_hi - head_lo
    dev = big0.device
    slab = [n * L * nh * d * elem for L in lengths]
    live = torch.tensor(lengths, dtype=torch.int64, device=dev)
    for part, head0 in ((0, head_lo), (1, hk + head_lo)):
        src = torch.tensor([big0.data_ptr() + (r * big0.stride(0) + head0 * d) * elem for r in rows],
                           dtype=torch.int64, device=dev)
        offs = torch.tensor([o + part * s for o, s in zip(dst_offsets, slab)], dtype=torch.int64,
                            device=dev)
        ops.kv_pack(src, live, offs, n, lstride, big0.stride(1) * elem, nh * d * elem,
                    max(lengths), dst)


def unpack_kv_heads(src, src_offsets: list[int], caches: dict, rows: list[int],
                    lengths: list[int], head_lo: int, head_hi: int):
    """Inverse of pack_kv_heads: scatters packed head slices into heads [head_lo, head_hi) of the
    live rows of requests `rows` of this all-layer cache."""
    from . import ops
    big0, n, lstride = _cache_geometry(caches)
    hk, d, elem = big0.shape[-2], big0.shape[-1], big0.element_size()
    if not 0 <= head_lo < head_hi <= hk:
        raise ValueError(f"head range [{head_lo}, {head_hi}) outside the cache's {hk} heads")
    nh = head_hi - head_lo
    dev = big0.device
    slab = [n * L * nh * d * elem for L in lengths]
    live = torch.tensor(lengths, dtype=torch.int64, device=dev)
    for part, head0 in ((0, head_lo), (1, hk + head_lo)):
        dst = torch.tensor([big0.data_ptr() + (r * big0.stride(0) + head0 * d) * elem for r in rows],
                           dtype=torch.int64, device=dev)
        offs = torch.tensor([o + part * s for o, s in zip(src_offsets, slab)], dtype=torch.int64,
                            device=dev)
        ops.kv_unpack(src, offs, live, dst, n, lstride, big0.stride(1) * elem, nh * d * elem,
                      max(lengths))


def reshard_kv(src_caches: list[dict], dst_caches: list[dict], rows: list[int],
               lengths: list[int], n_kv_heads: int):
    """Moves the live rows of requests `rows` from caches sharded over len(src_caches) TP ranks
    into caches sharded over len(dst_caches) ranks, all held by this process (one device or
    several): for every move of reshard_plan, one pack into a staging buffer on the source's
    device (launched with that device current, on its current stream) and one unpack into the
    destination with the destination's device current. When the two devices differ the staging
    buffer is first copied to the destination's device (torch orders that copy after the pack
    and before the unpack), so no kernel dereferences another GPU's memory. Across processes the
    same moves run with the staging buffer exposed through KVHandoff."""
    src_tp, dst_tp = len(src_caches), len(dst_caches)
    hs, hd = n_kv_heads // src_tp, n_kv_heads // dst_tp
    for s, t, lo, hi in reshard_plan(n_kv_heads, src_tp, dst_tp):
        nh = hi - lo
        sizes = head_slice_bytes(src_caches[s], lengths, nh)
        offs, o = [], 0
        for b in sizes:
            offs.append(o)
            o += (b + 15) // 16 * 16
        src_dev, dst_dev = src_caches[s][0].device, dst_caches[t][0].device
        with torch.cuda.device(src_dev):
            staging = torch.empty(max(o, 16), dtype=torch.uint8, device=src_dev)
            pack_kv_heads(src_caches[s], rows, lengths, lo - s * hs, hi - s * hs, staging, offs)
        with torch.cuda.device(dst_dev):
            if staging.device != dst_dev:
                staging = staging.to(dst_dev)
            unpack_kv_heads(staging, offs, dst_caches[t], rows, lengths, lo - t * hd, hi - t * hd)
