"""Device parity of the cache operations around the hot path:
snapshot / restore (QuantizedKVCache.swift:106-129), the continuous-batch
left-padded stack and scatter-back (BatchedDecode.swift:96-151,
ContinuousBatcher.swift:763-773), prefix store + fork with copy-on-write
(PrefixCache.swift:369-400, InferenceEngine.swift:1305-1417), and the NVLink
peer fetch of a prefix entry (two GPUs)."""
import math

import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, host_bits, prefill  # noqa: E402

D, HQ, HKV, LAYERS = 128, 32, 8, 2


def make(pool, rng, L, dtype=BF16):
    s = pool.create_sequence()
    k = to_bits(kv_values(rng, (LAYERS, HKV, L, D)), dtype)
    v = to_bits(kv_values(rng, (LAYERS, HKV, L, D)), dtype)
    prefill(pool, s, k, v, dtype)
    return s, k, v


def snap_np(snap):
    return (snap.keys.cpu().numpy(), snap.values.cpu().numpy(), host_bits(snap.key_scales),
            host_bits(snap.key_zeros), host_bits(snap.value_scales), host_bits(snap.value_zeros))


def attn(pool, seqs, q):
    out = torch.empty((LAYERS, len(seqs), HQ, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, seqs, 0, q, out, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    return out


def test_snapshot_restore_round_trip_does_not_alias():
    rng = np.random.default_rng(0)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=32)
    a, _, _ = make(pool, rng, 700)
    snap = a.quantized_snapshot(1)
    before = snap_np(snap)
    b = pool.create_sequence()
    b.restore_quantized(1, snap)
    assert b.length(1) == 700 and b.length(0) == 0
    got = snap_np(b.quantized_snapshot(1))
    for x, y in zip(got, before):
        np.testing.assert_array_equal(x, y)
    # truncate + update in place must not touch the source snapshot
    b.truncate(300)
    k1 = dev_bits(to_bits(kv_values(rng, (1, 1, HKV, 5, D)), BF16), BF16)
    kb.append_quantize(pool, [b], 1, k1, k1)
    torch.cuda.synchronize()
    for x, y in zip(snap_np(snap), before):
        np.testing.assert_array_equal(x, y)
    assert b.length(1) == 305
    pool.close()


def test_stack_left_padded_and_scatter_back():
    rng = np.random.default_rng(1)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=48)
    lens = [100, 350, 7]
    rows = [make(pool, rng, L) for L in lens]
    seqs = [r[0] for r in rows]
    s_max = max(lens)
    st = kb.stack_caches_left_padded_quantized(pool, seqs, 0)
    torch.cuda.synchronize()
    keys = st.keys.cpu().numpy()
    ks = host_bits(st.key_scales)
    for i, (s, k, _) in enumerate(rows):
        pad = s_max - lens[i]
        ck, sk, zk = oracle.quantize(k[0], BF16, 64)
        # pads: code 0, scale 0, zero 0 (dequantizes to exactly 0)
        assert (keys[i, :, :pad] == 0).all() and (ks[i, :, :pad] == 0).all()
        np.testing.assert_array_equal(keys[i, :, pad:], ck)
        np.testing.assert_array_equal(ks[i, :, pad:], sk)
    # an epoch of 3 "batched" steps grows the stacked layout by 3 columns;
    # scatter-back restores each row's own non-pad suffix
    steps = 3
    width = s_max + steps
    grown = [torch.zeros((len(seqs), HKV, width, D), dtype=torch.uint8, device="cuda")] + \
            [torch.zeros((len(seqs), HKV, width, 2), dtype=torch.float16, device="cuda") for _ in range(4)]
    grown = kb.QuantizedKVSnapshot(grown[0], grown[0].clone(), *grown[1:])
    grown.keys[:, :, :s_max] = st.keys
    grown.values[:, :, :s_max] = st.values
    for dst, src in zip([grown.key_scales, grown.key_zeros, grown.value_scales, grown.value_zeros],
                        [st.key_scales, st.key_zeros, st.value_scales, st.value_zeros]):
        dst[:, :, :s_max] = src
    extra = torch.randint(0, 256, (len(seqs), HKV, steps, D), dtype=torch.uint8, device="cuda")
    grown.keys[:, :, s_max:] = extra
    grown.values[:, :, s_max:] = extra
    for m in [grown.key_scales, grown.key_zeros, grown.value_scales, grown.value_zeros]:
        m[:, :, s_max:] = 0.5
    kb.scatter_back(pool, seqs, 0, grown, lens, s_max, steps)
    torch.cuda.synchronize()
    for i, s in enumerate(seqs):
        assert s.length(0) == lens[i] + steps
        sn = s.quantized_snapshot(0)
        np.testing.assert_array_equal(sn.keys.cpu().numpy(),
                                      grown.keys[i, :, s_max - lens[i]:].cpu().numpy())
        np.testing.assert_array_equal(host_bits(sn.value_zeros),
                                      host_bits(grown.value_zeros[i, :, s_max - lens[i]:]))
    pool.close()


def test_prefix_fork_cow_on_device():
    rng = np.random.default_rng(2)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=64)
    pc = kb.PrefixCache(pool)
    base, k, v = make(pool, rng, 600)
    toks = list(range(600))
    pc.store_quantized(toks, "m", base)
    q = dev_bits(to_bits(kv_values(rng, (LAYERS, 1, HQ, D)), BF16), BF16)
    want = attn(pool, [base], q)
    hit = pc.lookup_quantized(toks, "m")
    f1 = hit.fork(600)
    f2 = hit.fork(599)  # full hit: truncate(count - 1)
    hit.release()
    # the fork attends exactly the same blocks: bit-identical output
    assert torch.equal(attn(pool, [f1], q), want)
    # divergent appends into the shared partial last block -> COW each
    k1 = to_bits(kv_values(rng, (LAYERS, 1, HKV, 1, D)), BF16)
    k2 = to_bits(kv_values(rng, (LAYERS, 1, HKV, 1, D)), BF16)
    kb.append_quantize(pool, [f1], 0, dev_bits(k1, BF16), dev_bits(k1, BF16))
    kb.append_quantize(pool, [f2], 0, dev_bits(k2, BF16), dev_bits(k2, BF16))
    torch.cuda.synchronize()
    assert f1.blocks()[-1] != base.blocks()[-1] != f2.blocks()[-1]
    # the base (and the prefix entry) still attend their original data
    assert torch.equal(attn(pool, [base], q), want)
    # each fork's cache = prefix + its own token, checked against the oracle
    for f, kn, n in [(f1, k1, 600), (f2, k2, 599)]:
        for layer in range(LAYERS):
            kk = np.concatenate([k[layer][:, :n], kn[layer, 0]], axis=1)
            ck, _, _ = oracle.quantize(kk, BF16, 64)
            np.testing.assert_array_equal(f.quantized_snapshot(layer).keys.cpu().numpy(), ck)
    pool.close()


def test_prefix_peer_fetch_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rng = np.random.default_rng(3)
    p0 = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=32, device=0)
    p1 = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=32, device=1)
    pc0, pc1 = kb.PrefixCache(p0), kb.PrefixCache(p1)
    with torch.cuda.device(0):
        base, _, _ = make(p0, rng, 520)
        pc0.store_quantized(list(range(520)), "m", base)
        hit0 = pc0.lookup_quantized(list(range(520)), "m")
        q0 = dev_bits(to_bits(kv_values(rng, (LAYERS, 1, HQ, D)), BF16), BF16)
        want = attn(p0, [base], q0).cpu()
    with torch.cuda.device(1):
        stream = torch.cuda.current_stream()
        hit1 = pc1.peer_fetch(pc0, hit0, stream=stream)
        torch.cuda.synchronize()
        assert pc1.memory_count == 1
        f = hit1.fork(520)
        out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float32, device="cuda:1")
        kb.decode_attention(p1, [f], 0, q0.to("cuda:1"), out, 1 / math.sqrt(D))
        torch.cuda.synchronize()
        assert torch.equal(out.cpu(), want)
        # later lookups on GPU 1 hit locally
        local = pc1.lookup_quantized(list(range(520)), "m")
        assert local is not None and local.prefix_length == 520
        local.release()
        hit1.release()
    hit0.release()
    p0.close()
    p1.close()
