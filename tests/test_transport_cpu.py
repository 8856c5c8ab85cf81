"""Transport protocol on real 2-process Gloo groups (the reference's tests/test_transport.py
cases), the packed single-message layout, and header KATs from the reference."""
import json
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hexgen2_b200.transport import (recv_data, recv_packet, send_data, send_packet,
                                    validate_header)


def _worker(rank, rendezvous, packed):
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=2, init_method=Path(rendezvous).as_uri(),
                            timeout=timedelta(seconds=30))
    try:
        for dtype in (torch.float16, torch.bfloat16, torch.float32):
            cache = {7: torch.arange(-24, 24).reshape(1, 4, 2, 2, 3).to(dtype)[..., ::2],
                     2: torch.full((1, 3, 2, 1, 4), -1.25, dtype=dtype)}
            token = torch.tensor([42, 17], dtype=torch.long)
            if rank == 0:
                send_data(token, cache, dst=1, packed=packed)
                received, returned = recv_data(src=1, num_layers=2)
            else:
                received, returned = recv_data(src=0, num_layers=2)
                send_data(received, returned, dst=0, packed=packed)
            torch.testing.assert_close(received, token, rtol=0, atol=0)
            if list(returned) != [7, 2]:
                raise AssertionError("Layer IDs/order changed")
            for key in cache:
                torch.testing.assert_close(returned[key], cache[key], rtol=0, atol=0)
        # Empty tensors and metadata survive too.
        if rank == 0:
            n = send_packet({"e": torch.zeros(0, 3), "x": torch.ones(2)}, {"id": "a"}, dst=1,
                            packed=packed)
            assert n == 8
        else:
            t, meta = recv_packet(src=0)
            assert meta == {"id": "a"} and t["e"].shape == (0, 3) and t["x"].tolist() == [1, 1]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("packed", [False, True])
def test_lossless_real_process_roundtrip(tmp_path, packed):
    mp.spawn(_worker, args=(str(tmp_path / "rendezvous"), packed), nprocs=2, join=True)


def test_invalid_metadata_is_rejected_before_allocating_payload():
    for shape in ([-1], [True], [2 ** 40], [1] * 9):
        with pytest.raises(ValueError):
            validate_header({"version": 1, "tensors": [{"name": "x", "shape": shape,
                                                        "dtype": "torch.float32"}]})
    with pytest.raises(ValueError):
        validate_header({"version": 1, "tensors": [
            {"name": "x", "shape": [1], "dtype": "torch.float32"},
            {"name": "x", "shape": [1], "dtype": "torch.float32"}]})
    with pytest.raises(ValueError):
        validate_header({"version": 2, "tensors": []})
    with pytest.raises(ValueError):
        validate_header({"version": 1, "tensors": [{"name": "x", "shape": [1], "dtype": "float"}]})
    with pytest.raises(ValueError):
        validate_header({"version": 1, "tensors": [{"name": str(i), "shape": [1],
                                                    "dtype": "torch.uint8"} for i in range(1025)]})


def test_header_bytes_match_reference(golden):
    """The header JSON we send is byte-identical to the reference's for the pilot packet."""
    for p in golden["transport"]:
        h = p["header"]
        assert validate_header(h) == p["payload_bytes"]
        assert json.dumps(h, allow_nan=False) == p["header_utf8"]


def _fault_worker(rank, rendezvous):
    dist.init_process_group("gloo", rank=rank, world_size=2, init_method=Path(rendezvous).as_uri(),
                            timeout=timedelta(seconds=30))
    try:
        if rank == 0:
            # A truncated/bogus header length: the receiver must raise before allocating.
            dist.send(torch.tensor([0], dtype=torch.int64), dst=1)
            dist.send(torch.tensor([2 * 1024 * 1024], dtype=torch.int64), dst=1)
        else:
            for _ in range(2):
                try:
                    recv_packet(src=0)
                    raise AssertionError("bad header accepted")
                except ValueError:
                    pass
    finally:
        dist.destroy_process_group()


def test_bad_header_length_rejected_on_real_ranks(tmp_path):
    mp.spawn(_fault_worker, args=(str(tmp_path / "rv"),), nprocs=2, join=True)


@pytest.mark.parametrize("heads,src,dst", [(8, 2, 4), (8, 4, 2), (8, 2, 1), (8, 1, 8), (32, 4, 2), (6, 3, 2)])
def test_reshard_plan_covers_every_head_once(heads, src, dst):
    from hexgen2_b200.transport import reshard_plan
    plan = reshard_plan(heads, src, dst)
    seen = []
    for s, t, lo, hi in plan:
        assert s * (heads // src) <= lo < hi <= (s + 1) * (heads // src)  # inside the source shard
        assert t * (heads // dst) <= lo < hi <= (t + 1) * (heads // dst)  # inside the dest shard
        seen.extend(range(lo, hi))
    assert sorted(seen) == list(range(heads))
    assert [p[1] for p in plan] == sorted(p[1] for p in plan)


def test_reshard_plan_rejects_indivisible_sizes():
    from hexgen2_b200.transport import reshard_plan
    with pytest.raises(ValueError):
        reshard_plan(8, 3, 2)
    with pytest.raises(ValueError):
        reshard_plan(8, 2, 0)


REF_TRANSPORT = Path("/root/reference/hexgen2/transport.py")


def _load_reference_transport():
    import importlib.util
    spec = importlib.util.spec_from_file_location("_ref_transport", REF_TRANSPORT)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _interop_worker(rank, rendezvous):
    """Rank 0 runs this package's transport, rank 1 the reference's own module (imported
    unchanged from its source file); packets go both ways for every KV dtype."""
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=2, init_method=Path(rendezvous).as_uri(),
                            timeout=timedelta(seconds=30))
    try:
        ref = _load_reference_transport()
        for dtype in (torch.float16, torch.bfloat16, torch.float32):
            # A prefill result as this package returns it: per-layer contiguous views of ONE
            # packed buffer ([1, L, 2, hkv, d] each), plus the first token.
            L, layers, hk, d = 5, 3, 2, 8
            buf = torch.arange(layers * L * 2 * hk * d, dtype=torch.float32).to(dtype)
            view = buf.view(layers, 1, L, 2, hk, d)
            cache = {i: view[i] for i in range(layers)}
            token = torch.tensor([123], dtype=torch.long)
            if rank == 0:
                n = send_data(token, cache, dst=1)                       # ours -> reference
                assert n == 8 + layers * L * 2 * hk * d * buf.element_size()
                got_tok, got = recv_data(src=1, num_layers=layers)      # reference -> ours
            else:
                got_tok, got = ref.recv_data(src=0, num_layers=layers)
                ref.send_data(got_tok, got, dst=0)
            assert torch.equal(got_tok, token)
            assert list(got) == list(range(layers))
            for i in range(layers):
                assert got[i].dtype == dtype and torch.equal(got[i], cache[i]), (dtype, i)
        # Metadata and empty tensors, reference sender -> this receiver.
        if rank == 1:
            ref.send_packet({"e": torch.zeros(0, 3), "x": torch.ones(2, dtype=torch.int32)},
                            {"request": "r-1", "layers": []}, dst=0)
        else:
            t, meta = recv_packet(src=1)
            assert meta == {"request": "r-1", "layers": []}
            assert t["e"].shape == (0, 3) and t["x"].dtype == torch.int32
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not REF_TRANSPORT.exists(), reason="reference sources not mounted")
def test_interop_with_reference_transport(tmp_path):
    """This package's send_packet/send_data feed the reference's recv_packet/recv_data and the
    reverse (hexgen2/transport.py:44-100), on a real 2-process Gloo group."""
    mp.spawn(_interop_worker, args=(str(tmp_path / "rendezvous"),), nprocs=2, join=True)


def test_cache_geometry_and_head_slice_bytes():
    """The re-shard path's host checks: an engine cache is one all-layer tensor handed out as
    per-layer views at a fixed stride, and a head slice's packed size is K + V slabs of every
    layer; views not at one fixed stride and rows that are not contiguous are rejected."""
    from hexgen2_b200.transport import _cache_geometry, head_slice_bytes
    layers, B, cap, hk, d = 3, 2, 16, 4, 8
    big = torch.zeros(layers, B, cap, 2, hk, d, dtype=torch.bfloat16)
    caches = {i: big[i] for i in range(layers)}
    base, n, stride = _cache_geometry(caches)
    assert base.data_ptr() == big.data_ptr() and n == layers
    assert stride == B * cap * 2 * hk * d * 2
    assert head_slice_bytes(caches, [5, 9], 2) == [2 * layers * 5 * 2 * d * 2,
                                                   2 * layers * 9 * 2 * d * 2]
    with pytest.raises(ValueError):  # layers out of order: not one strided region
        _cache_geometry({0: big[0], 1: big[2], 2: big[1]})
    with pytest.raises(ValueError):
        _cache_geometry({i: big[i].transpose(-1, -2) for i in range(layers)})
