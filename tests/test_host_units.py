"""Unit tests of the host runtime's building blocks (mirror the reference's
inline unit tests: codec.rs, header.rs, types.rs, reduce.rs, buffer_pool.rs,
compression/*.rs, sparse.rs, topology.rs, hash.rs, config.rs)."""
import os

import numpy as np
import pytest

from nexar_b200 import _native
from nexar_b200.core import DataType, ReduceOp

H = _native.host()


# ------------------------------------------------------------ wire
def test_header_roundtrip_and_layout():
    b = H.encode_header(0x01020304, 2, 0)
    assert b == bytes([4, 3, 2, 1, 2, 0, 0, 0])
    assert H.decode_header(b) == (0x01020304, 2, 0)
    assert H.decode_header(bytes([0, 0, 0, 0, 0, 9, 0, 0])) is None  # unknown message type


def test_every_message_variant_roundtrips():
    ok, total = H.message_roundtrip_selftest()
    assert ok == total == 17


def test_decode_rejects_truncated_and_trailing():
    from nexar_b200.core import DecodeFailed
    b = H.encode_barrier(5, 7, 0)
    d = H.decode_message(b)
    assert d["kind"] == "Barrier" and d["epoch"] == 5 and d["comm_id"] == 7
    with pytest.raises(DecodeFailed):
        H.decode_message(b[:-1])
    with pytest.raises(DecodeFailed):
        H.decode_message(b + b"\0")
    with pytest.raises(DecodeFailed):
        H.decode_message(b[:4])


def test_data_message_payload():
    d = H.decode_message(H.encode_data(9, 3, b"payload"))
    assert (d["kind"], d["tag"], d["src_rank"], d["payload"]) == ("Data", 9, 3, b"payload")


# ------------------------------------------------------------ reduce engine
@pytest.mark.parametrize("dt,np_t", [(DataType.F32, np.float32), (DataType.F64, np.float64),
                                     (DataType.I32, np.int32), (DataType.I64, np.int64),
                                     (DataType.U8, np.uint8), (DataType.I8, np.int8),
                                     (DataType.U32, np.uint32), (DataType.U64, np.uint64)])
@pytest.mark.parametrize("op", ["sum", "prod", "min", "max"])
def test_reduce_slice_matches_numpy(dt, np_t, op):
    rs = np.random.RandomState(1)
    if np.issubdtype(np_t, np.floating):
        a, b = rs.randn(1001).astype(np_t), rs.randn(1001).astype(np_t)
    else:
        info = np.iinfo(np_t)
        a = rs.randint(max(info.min, -1000), min(info.max, 1000), 1001).astype(np_t)
        b = rs.randint(max(info.min, -1000), min(info.max, 1000), 1001).astype(np_t)
    want = {"sum": np.add, "prod": np.multiply, "min": np.minimum, "max": np.maximum}[op](a, b)
    d = a.copy()
    H.reduce_slice(d.ctypes.data, b.ctypes.data, d.size, int(dt), int(ReduceOp.parse(op)))
    np.testing.assert_array_equal(d, want.astype(np_t))  # integer ops wrap like numpy


def test_bf16_round_to_nearest_even():
    import torch
    xs = torch.randn(10000, dtype=torch.float32) * 100
    for x in xs[:2000].tolist():
        assert H.f32_to_bf16(x) == torch.tensor([x]).to(torch.bfloat16).view(torch.int16).item() & 0xFFFF
    # exact tie: 1 + 2^-8 lies halfway between bf16 neighbours; even mantissa wins
    assert H.bf16_to_f32(H.f32_to_bf16(1.00390625)) == 1.0


def test_f16_conversion_matches_numpy():
    rs = np.random.RandomState(3)
    vals = np.concatenate([rs.randn(5000) * 10, rs.randn(1000) * 1e-5, [65504.0, 65520.0, 1e9, -1e-8, 0.0]])
    for v in vals.astype(np.float32):
        with np.errstate(over="ignore"):
            want = np.array([v], np.float32).astype(np.float16).view(np.uint16)[0]
        assert H.f32_to_f16(float(v)) == want, v
        assert H.f16_to_f32(int(want)) == float(np.array([want], np.uint16).view(np.float16)[0].astype(np.float32))


def test_bf16_f16_reduce_and_identity():
    import torch
    a = torch.randn(300).to(torch.bfloat16)
    b = torch.randn(300).to(torch.bfloat16)
    d = a.clone()
    H.reduce_slice(d.data_ptr(), b.data_ptr(), 300, int(DataType.BF16), 0)
    assert torch.equal(d, (a.float() + b.float()).to(torch.bfloat16))
    x = np.zeros(4, np.float32)
    H.fill_identity(x.ctypes.data, 4, int(DataType.F32), int(ReduceOp.Max))
    assert (x == np.finfo(np.float32).min).all()
    y = torch.zeros(4, dtype=torch.bfloat16)
    H.fill_identity(y.data_ptr(), 4, int(DataType.BF16), int(ReduceOp.Min))
    assert torch.isinf(y).all() and (y > 0).all()
    z = np.zeros(4, np.int8)
    H.fill_identity(z.ctypes.data, 4, int(DataType.I8), int(ReduceOp.Max))
    assert (z == -128).all()


def test_simd_path_reported():
    assert H.simd_path() in ("avx512f", "avx2", "scalar")


# ------------------------------------------------------------ comm ids
def test_fnv1a_comm_id():
    assert H.fnv1a_comm_id([b"\x01" + b"\0" * 7]) == H.fnv1a_comm_id([b"\x01" + b"\0" * 7])
    assert H.fnv1a_comm_id([b"a"]) != H.fnv1a_comm_id([b"b"])
    assert H.fnv1a_comm_id([]) == 0xcbf29ce484222325
    assert all(H.fnv1a_comm_id([i.to_bytes(8, "little")]) != 0 for i in range(1000))


# ------------------------------------------------------------ buffer pool
def test_buffer_pool_tiers_and_reuse():
    pool = H.BufferPool.with_config(4, 1024)
    b = pool.checkout(100)
    assert b.size == 100 and b.tobytes() == b"\0" * 100 and b.tier == 0
    del b
    assert pool.free_count(0) == 1
    p2 = H.BufferPool.with_profile(0)
    for size, tier in [(100, 0), (1 << 20, 1), (32 << 20, 2), (128 << 20, 3), (512 << 20, 4)]:
        assert p2.tier_for_size(size) == tier
    small = H.BufferPool.with_config(1, 64)
    b1, b2 = small.checkout(10), small.checkout(10)
    del b1, b2  # second return finds the tier full and is dropped
    assert small.free_count(0) == 1


# ------------------------------------------------------------ compressors
def test_compressed_tensor_format_and_topk_selection():
    x = np.array([0.1, -5.0, 0.2, 3.0, -0.05, 4.0], np.float32)
    res = np.zeros_like(x)
    ct = H.TopKCompressor(0.5).compress(x.ctypes.data, 6, int(DataType.F32), res.ctypes.data)
    assert ct.k == 3 and ct.indices == [1, 3, 5]
    raw = ct.data
    assert int.from_bytes(raw[:4], "little") == 3
    vals = np.frombuffer(raw[4 + 12:], np.float32)
    np.testing.assert_array_equal(vals, [-5.0, 3.0, 4.0])
    np.testing.assert_array_equal(res, np.array([0.1, 0, 0.2, 0, -0.05, 0], np.float32))
    out = np.zeros(6, np.float32)
    H.TopKCompressor(0.5).decompress(raw, 6, int(DataType.F32), out.ctypes.data)
    np.testing.assert_array_equal(out, [0, -5.0, 0, 3.0, 0, 4.0])


def test_topk_bf16_and_randomk_deterministic():
    import torch
    x = torch.tensor([0.5, -8.0, 1.0, 2.0], dtype=torch.bfloat16)
    r = torch.zeros(4, dtype=torch.bfloat16)
    ct = H.TopKCompressor(0.5).compress(x.data_ptr(), 4, int(DataType.BF16), r.data_ptr())
    assert ct.indices == [1, 3]
    a = np.arange(100, dtype=np.float32)
    r1, r2 = np.zeros(100, np.float32), np.zeros(100, np.float32)
    c1 = H.RandomKCompressor(0.1).compress(a.ctypes.data, 100, 0, r1.ctypes.data)
    c2 = H.RandomKCompressor(0.1).compress(a.ctypes.data, 100, 0, r2.ctypes.data)
    assert c1.indices == c2.indices and c1.k == 10 and len(set(c1.indices)) == 10
    nc = H.NoCompression().compress(a.ctypes.data, 100, 0, r1.ctypes.data)
    assert nc.k == 100


# ------------------------------------------------------------ topology
def test_topology_neighbors():
    assert H.build_neighbors("full_mesh", 0, 4) == [1, 2, 3]
    assert H.build_neighbors("k_regular:4", 0, 8) == [1, 2, 6, 7]
    assert H.build_neighbors("k_regular:4", 7, 8) == [0, 1, 5, 6]
    assert H.build_neighbors("hypercube", 0, 8) == [1, 2, 4]
    assert H.build_neighbors("hypercube", 5, 8) == [1, 4, 7]


def test_routing_tables():
    nb, hops = H.build_routing_table("k_regular:4", 0, 16)
    assert nb == [1, 2, 14, 15]
    assert hops[5] in nb
    nb, hops = H.build_routing_table("hypercube", 0, 8)
    assert hops[7] == 4 and hops[3] == 2
    nb, hops = H.build_routing_table("full_mesh", 0, 8)
    assert hops == {}


def test_spanning_tree_covers_all():
    parent, children = H.build_spanning_tree("k_regular:4", 0, 16)
    assert len(parent) == 15 and 0 not in parent
    reach = {0}
    frontier = [0]
    while frontier:
        n = frontier.pop()
        for ch in children[n]:
            reach.add(ch)
            frontier.append(ch)
    assert reach == set(range(16))


def test_alternative_hop_and_parse():
    alt = H.find_alternative_hop("hypercube", 0, 7, 4, 8)
    assert alt in (1, 2)
    assert H.optimal_ring_order(4) == [0, 1, 2, 3]
    assert str(H.parse_topology("k_regular:6")) == "k_regular:6"
    with pytest.raises(Exception):
        H.parse_topology("bogus")


def test_cluster_map():
    m = H.ClusterMap()
    m.add_peer(0, "a:1")
    m.add_peer(1, "b:2")
    m.heartbeat(0, 10.0)
    m.heartbeat(1, 1.0)
    e0 = m.epoch
    assert m.check_timeouts(12.0, 5.0) == [1]
    assert m.alive_peers() == [0] and m.epoch > e0
    m.remove_peer(1)
    assert m.size() == 1 and not m.contains(1) and m.addr(0) == "a:1"


# ------------------------------------------------------------ config
def test_config_defaults_and_env(monkeypatch):
    c = H.Config()
    assert c.collective_timeout_s == 30 and c.large_msg_bytes == 8 << 20
    assert c.pipeline_segment_bytes == 2 << 20 and c.ring_max_world == 8
    assert c.heartbeat_interval_s == 1 and c.heartbeat_timeout_s == 5
    assert c.compressed_allreduce_max_bytes == 4 << 30 and c.topology == "full_mesh"
    monkeypatch.setenv("NEXAR_COLLECTIVE_TIMEOUT_SECS", "7")
    monkeypatch.setenv("NEXAR_TOPOLOGY", "hypercube")
    monkeypatch.setenv("NEXAR_RECOVERY_POLICY", "abort")
    monkeypatch.setenv("NEXAR_RING_MAX_WORLD", "3")
    e = H.Config.from_env()
    assert e.collective_timeout_s == 7 and e.topology == "hypercube" and e.recovery_policy == 2
    assert e.ring_max_world == 3


def test_memory_buffer_refs_and_pool_builder():
    """BufferRef memory-space markers and the pool builder (nexar/src/memory/buffer.rs,
    transport/buffer_pool.rs)."""
    import numpy as np
    import torch
    from nexar_b200.core import DataType
    from nexar_b200.memory import BufferPool, BufferRef, Device, Host, PoolBuilder, PoolProfile, TierConfig
    a = np.zeros(12, np.float32)
    r = BufferRef.host(a)
    assert r.space is Host and r.len_bytes() == 48 and r.count() == 12 and r.as_u64() == a.ctypes.data
    assert r.dtype == DataType.F32 and not r.is_empty()
    t = torch.zeros(5, dtype=torch.bfloat16)
    assert BufferRef(t).len_bytes() == 10 and BufferRef(t).space is Host
    with pytest.raises(ValueError):
        BufferRef.device(t)  # a CPU tensor is host memory
    raw = BufferRef(address=0x1000, nbytes=64, dtype=DataType.F64, space=Device)
    assert raw.count() == 8 and raw.ptr().space is Device
    pool = PoolBuilder().small(TierConfig(2, 1024)).large(TierConfig(1, 1 << 20)).build()
    b = pool.checkout(100)
    assert b.size == 100 and b.tier == 0
    assert pool.tier_for_size(2000) == 1
    assert BufferPool.with_profile(PoolProfile.Inference).free_count(0) >= 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("op", [0, 1, 2, 3])  # Sum, Prod, Min, Max
def test_half_reduce_vector_paths_match_scalar_definition(dtype, op):
    """The SIMD bf16 / f16 reductions (16 or 8 lanes wide plus a scalar tail)
    agree bit for bit with the scalar conversion rules on every class of
    input: normals, subnormals, +-0, +-inf, NaN (any NaN matches any NaN)."""
    import numpy as np
    H = _native.host()
    rs = np.random.RandomState(op * 7 + (dtype == "f16"))
    n = 4099  # vector blocks and a tail
    a = rs.randint(0, 1 << 16, n).astype(np.uint16)
    b = rs.randint(0, 1 << 16, n).astype(np.uint16)
    # special values in both operands
    if dtype == "bf16":
        specials = [0x0000, 0x8000, 0x7f80, 0xff80, 0x7fc1, 0x0001, 0x8001, 0x3f80, 0x7f7f]
    else:
        specials = [0x0000, 0x8000, 0x7c00, 0xfc00, 0x7e01, 0x0001, 0x8001, 0x3c00, 0x7bff]
    a[:len(specials)] = specials
    b[len(specials):2 * len(specials)] = specials
    to_f = H.bf16_to_f32 if dtype == "bf16" else H.f16_to_f32
    from_f = H.f32_to_bf16 if dtype == "bf16" else H.f32_to_f16
    fns = [lambda x, y: x + y, lambda x, y: x * y, lambda x, y: y if y < x else x, lambda x, y: y if y > x else x]
    with np.errstate(all="ignore"):  # inf / NaN results are part of the test
        want = np.array([from_f(float(np.float32(fns[op](np.float32(to_f(int(x))), np.float32(to_f(int(y)))))))
                         for x, y in zip(a, b)], np.uint16)
    got = a.copy()
    code = DataType.BF16 if dtype == "bf16" else DataType.F16
    H.reduce_slice(got.ctypes.data, b.ctypes.data, n, int(code), op)
    if dtype == "bf16":
        is_nan = lambda v: ((v & 0x7f80) == 0x7f80) & ((v & 0x007f) != 0)
    else:
        is_nan = lambda v: ((v & 0x7c00) == 0x7c00) & ((v & 0x03ff) != 0)
    both_nan = is_nan(got) & is_nan(want)
    mism = (got != want) & ~both_nan
    assert not mism.any(), [(int(a[i]), int(b[i]), int(got[i]), int(want[i])) for i in np.nonzero(mism)[0][:5]]


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.float16])
@pytest.mark.parametrize("n,ratio", [(1, 0.5), (7, 0.3), (10_003, 0.01), (10_003, 0.999), (10_003, 1.0), (4096, 0.25)])
def test_topk_selection_matches_sort_reference(dtype, n, ratio):
    """The radix-select top-k equals a full sort by (|r| desc, index asc) for
    random data with many repeated magnitudes, odd lengths, k = 1 .. n."""
    import math
    code = {np.float32: DataType.F32, np.float64: DataType.F64, np.float16: DataType.F16}[dtype]
    rs = np.random.RandomState(n + int(ratio * 1000))
    x = (rs.randint(-40, 41, n) / 8.0).astype(dtype)  # few distinct magnitudes: ties everywhere
    res = (rs.randn(n) * (rs.rand(n) < 0.5)).astype(dtype)
    r_before = (res.astype(np.float64) + x.astype(np.float64)).astype(dtype)  # residual += input
    k = max(1, math.ceil(n * ratio))
    mag = np.abs(r_before.astype(np.float32))
    order = np.lexsort((np.arange(n), -mag))  # magnitude desc, then index asc
    want = np.sort(order[:k])
    ct = H.TopKCompressor(ratio).compress(x.ctypes.data, n, int(code), res.ctypes.data)
    assert ct.k == k
    assert ct.indices == want.tolist()
    left = r_before.copy()
    left[want] = 0
    np.testing.assert_array_equal(res, left)
