"""Decode step from host buffers (krill_decode_step_host): the layers run in
chunks with their input and output copies overlapped on side streams. With a
fixed split length a (layer, sequence) result does not depend on the rest of
the call, so every chunking must give bit-identical outputs and cache
contents to krill_decode_step on device buffers (itself checked against the
oracle in test_gpu_attention.py)."""
import numpy as np
import pytest

from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import TORCH16, dev_bits, prefill  # noqa: E402


def host_tensor(bits: np.ndarray, dtype: int, pinned: bool) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TORCH16[dtype])
    return t.pin_memory() if pinned else t.clone()


def twin_pools(layers, hkv, hq, D, lengths, dtype, rng):
    pools = [kb.KVPool(layers, hkv, hq, D, num_blocks=64, group_size=64, split_tokens=256)
             for _ in range(2)]
    seqs = [[], []]
    for L in lengths:
        k = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        for i in range(2):
            s = pools[i].create_sequence()
            prefill(pools[i], s, k, v, dtype)
            seqs[i].append(s)
    return pools, seqs


@pytest.mark.parametrize("chunk,pinned,out_f32", [(0, True, False), (1, True, False), (4, True, True),
                                                  (6, False, False), (3, False, True)])
def test_host_step_matches_device_step(chunk, pinned, out_f32):
    layers, hkv, hq, D, dtype = 6, 4, 16, 128, BF16
    rng = np.random.default_rng(7 + chunk)
    lengths = [300, 1, 777, 2049]
    (pa, pb), (sa, sb) = twin_pools(layers, hkv, hq, D, lengths, dtype, rng)
    n = len(lengths)
    odt = torch.float32 if out_f32 else TORCH16[dtype]
    stream = torch.cuda.current_stream()
    for step in range(3):
        k1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
        v1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
        qb = to_bits(kv_values(rng, (layers, n, hq, D)), dtype)
        out_dev = torch.empty((layers, n, hq, D), dtype=odt, device="cuda")
        kb.decode_step(pa, sa, 0, dev_bits(k1, dtype), dev_bits(v1, dtype), dev_bits(qb, dtype), out_dev,
                       0.088, stream=stream)
        out_host = torch.empty((layers, n, hq, D), dtype=odt, pin_memory=pinned)
        out_host.fill_(float("nan"))
        kb.decode_step_host(pb, sb, 0, host_tensor(k1, dtype, pinned), host_tensor(v1, dtype, pinned),
                            host_tensor(qb, dtype, pinned), out_host, 0.088, layer_chunk=chunk,
                            stream=stream)
        stream.synchronize()
        a = out_dev.cpu().view(torch.int32 if out_f32 else torch.int16)
        b = out_host.view(torch.int32 if out_f32 else torch.int16)
        assert torch.equal(a, b), f"step {step}: host-buffer step differs from the device step"
    for i in range(n):
        for layer in range(layers):
            assert sa[i].length(layer) == sb[i].length(layer) == lengths[i] + 3
    assert pa.device_error() == 0 and pb.device_error() == 0


def test_host_step_layer_subrange_and_errors():
    layers, hkv, hq, D, dtype = 4, 2, 8, 64, F16
    rng = np.random.default_rng(3)
    (pa, pb), (sa, sb) = twin_pools(layers, hkv, hq, D, [129, 640], dtype, rng)
    n = 2
    k1 = to_bits(kv_values(rng, (2, n, hkv, 1, D)), dtype)
    v1 = to_bits(kv_values(rng, (2, n, hkv, 1, D)), dtype)
    qb = to_bits(kv_values(rng, (2, n, hq, D)), dtype)
    out_dev = torch.empty((2, n, hq, D), dtype=torch.float16, device="cuda")
    kb.decode_step(pa, sa, 1, dev_bits(k1, dtype), dev_bits(v1, dtype), dev_bits(qb, dtype), out_dev, 0.125)
    out_host = torch.empty((2, n, hq, D), dtype=torch.float16, pin_memory=True)
    kb.decode_step_host(pb, sb, 1, host_tensor(k1, dtype, True), host_tensor(v1, dtype, True),
                        host_tensor(qb, dtype, True), out_host, 0.125, layer_chunk=1)
    torch.cuda.synchronize()
    assert torch.equal(out_dev.cpu().view(torch.int16), out_host.view(torch.int16))
    assert [s.length(0) for s in sb] == [129, 640] and [s.length(1) for s in sb] == [130, 641]
    with pytest.raises(ValueError):
        kb.decode_step_host(pb, sb, 1, dev_bits(k1, dtype), host_tensor(v1, dtype, True),
                            host_tensor(qb, dtype, True), out_host, 0.125)
    with pytest.raises(kb.KrillError):
        kb.decode_step_host(pb, sb, 3, host_tensor(k1, dtype, True), host_tensor(v1, dtype, True),
                            host_tensor(qb, dtype, True), out_host, 0.125)


@pytest.mark.parametrize("chunk", [0, 1])
def test_host_step_sliding_window_pool(chunk):
    """A sliding-window pool (ring of blocks, RotatingKVCache semantics):
    the host-buffer step must match the device step bit for bit while the
    ring wraps."""
    layers, hkv, hq, D, dtype, window = 2, 4, 8, 256, F16, 128
    rng = np.random.default_rng(21 + chunk)
    lengths = [10, 300, 700]
    pools = [kb.KVPool(layers, hkv, hq, D, num_blocks=32, group_size=64, window=window, split_tokens=256)
             for _ in range(2)]
    seqs = [[], []]
    for L in lengths:
        k = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        for i in range(2):
            s = pools[i].create_sequence()
            prefill(pools[i], s, k, v, dtype, chunk=256)
            seqs[i].append(s)
    (pa, pb), (sa, sb) = pools, seqs
    n = len(lengths)
    for step in range(3):
        k1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
        v1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
        qb = to_bits(kv_values(rng, (layers, n, hq, D)), dtype)
        out_dev = torch.empty((layers, n, hq, D), dtype=torch.float16, device="cuda")
        kb.decode_step(pa, sa, 0, dev_bits(k1, dtype), dev_bits(v1, dtype), dev_bits(qb, dtype), out_dev, 1.0)
        out_host = torch.empty((layers, n, hq, D), dtype=torch.float16, pin_memory=True)
        out_host.fill_(float("nan"))
        kb.decode_step_host(pb, sb, 0, host_tensor(k1, dtype, True), host_tensor(v1, dtype, True),
                            host_tensor(qb, dtype, True), out_host, 1.0, layer_chunk=chunk)
        torch.cuda.synchronize()
        assert torch.equal(out_dev.cpu().view(torch.int16), out_host.view(torch.int16)), f"step {step}"
    assert [s.length(0) for s in sb] == [L + 3 for L in lengths]
    assert pa.device_error() == 0 and pb.device_error() == 0


def test_host_step_shared_prefix_cascade():
    """Forks of one prefix-cache entry attend the shared blocks through the
    tcgen05 cascade kernel, which then reads the query from mapped host
    memory too; the host step must match the device step bit for bit."""
    layers, hkv, hq, D, dtype = 2, 8, 32, 128, BF16
    rng = np.random.default_rng(11)
    P, suffixes = 1024, [5, 70, 300, 1]
    kp = to_bits(kv_values(rng, (layers, hkv, P, D)), dtype)
    vp = to_bits(kv_values(rng, (layers, hkv, P, D)), dtype)
    ks = [to_bits(kv_values(rng, (layers, hkv, S, D)), dtype) for S in suffixes]
    vs = [to_bits(kv_values(rng, (layers, hkv, S, D)), dtype) for S in suffixes]
    pools, seqs = [], []
    for _ in range(2):
        pool = kb.KVPool(layers, hkv, hq, D, num_blocks=64, group_size=64)
        pc = kb.PrefixCache(pool)
        base = pool.create_sequence()
        prefill(pool, base, kp, vp, dtype)
        toks = list(range(P))
        pc.store_quantized(toks, "m", base)
        base.release()
        hit = pc.lookup_quantized(toks, "m")
        ss = []
        for k, v in zip(ks, vs):
            f = hit.fork(P)
            prefill(pool, f, k, v, dtype)
            ss.append(f)
        hit.release()
        pools.append((pool, pc))
        seqs.append(ss)
    n = len(suffixes)
    (pa, _), (pb, _) = pools
    for step in range(2):
        k1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
        v1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
        qb = to_bits(kv_values(rng, (layers, n, hq, D)), dtype)
        out_dev = torch.empty((layers, n, hq, D), dtype=torch.bfloat16, device="cuda")
        kb.decode_step(pa, seqs[0], 0, dev_bits(k1, dtype), dev_bits(v1, dtype), dev_bits(qb, dtype),
                       out_dev, 0.088)
        assert pa.last_cascade()[0] >= 1, "the forks should form a cascade group"
        out_host = torch.empty((layers, n, hq, D), dtype=torch.bfloat16, pin_memory=True)
        kb.decode_step_host(pb, seqs[1], 0, host_tensor(k1, dtype, True), host_tensor(v1, dtype, True),
                            host_tensor(qb, dtype, True), out_host, 0.088)
        torch.cuda.synchronize()
        assert pb.last_cascade()[0] >= 1
        assert torch.equal(out_dev.cpu().view(torch.int16), out_host.view(torch.int16)), f"step {step}"
    assert pa.device_error() == 0 and pb.device_error() == 0


def test_decode_step_keeps_its_append_when_attention_fails():
    """krill_decode_step carries the append's destinations in the attention's
    metadata upload. When the attention call then fails (here: an invalid
    output dtype, rejected before any launch), the append is still uploaded
    and launched on its own: the cache must equal a twin pool that appended
    the same token normally, bit for bit."""
    import ctypes as C
    from krill_b200 import _lib as L
    layers, hkv, hq, D, dtype = 2, 8, 32, 128, BF16
    rng = np.random.default_rng(21)
    (pa, pb), (sa, sb) = twin_pools(layers, hkv, hq, D, [300, 1000], dtype, rng)
    n = 2
    k1 = dev_bits(to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype), dtype)
    v1 = dev_bits(to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype), dtype)
    q = dev_bits(to_bits(kv_values(rng, (layers, n, hq, D)), dtype), dtype)
    out = torch.empty((layers, n, hq, D), dtype=torch.float32, device="cuda")
    arr = (C.c_uint64 * n)(*[s.handle for s in sa])
    st = L.lib.krill_decode_step(pa.handle, n, arr, 0, layers, k1.data_ptr(), v1.data_ptr(), L.DTYPE_BF16,
                                 q.data_ptr(), L.DTYPE_BF16, out.data_ptr(), 9, 0.088, None)
    assert st == L.KRILL_ERR_INVALID
    kb.append_quantize(pb, sb, 0, k1, v1)
    torch.cuda.synchronize()
    for a, b in zip(sa, sb):
        for layer in range(layers):
            assert a.length(layer) == b.length(layer)
    oa, ob = torch.empty_like(out), torch.empty_like(out)
    kb.decode_attention(pa, sa, 0, q, oa, 0.088)
    kb.decode_attention(pb, sb, 0, q, ob, 0.088)
    torch.cuda.synchronize()
    assert torch.equal(oa.cpu().view(torch.int32), ob.cpu().view(torch.int32))
    assert pa.device_error() == 0 and pb.device_error() == 0
