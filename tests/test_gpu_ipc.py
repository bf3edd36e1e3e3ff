"""Cross-process NVLink fetch of a prefix entry (one process per GPU): the
owner publishes its pool's IPC handle and an entry descriptor, a process on
another GPU imports the entry into its own pool; attention over a fork of the
imported entry is bit-identical to the owner's. Needs two GPUs."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

D, HQ, HKV, LAYERS, S = 128, 32, 8, 2, 600


def _importer(q_in, q_out):
    """Child process on GPU 1: import the entry, attend a fork of it."""
    import torch
    import krill_b200 as kb
    torch.cuda.set_device(1)
    handle, desc, qbytes = q_in.get(timeout=120)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=16, device=1)
    pc = kb.PrefixCache(pool)
    stream = torch.cuda.current_stream()
    hit = pc.import_entry(handle, desc, stream=stream)
    torch.cuda.synchronize()
    q_out.put(("copied", hit.prefix_length))
    f = hit.fork(S)
    q = torch.frombuffer(bytearray(qbytes), dtype=torch.bfloat16).reshape(LAYERS, 1, HQ, D).cuda()
    out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, [f], 0, q, out, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    q_out.put(("out", out.cpu().numpy().tobytes(), pool.device_error()))
    hit.release()
    pc.close()
    pool.close()


def test_prefix_import_across_processes():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import krill_b200 as kb
    from tests._data import BF16, kv_values, to_bits
    from tests._gpu import dev_bits, prefill
    rng = np.random.default_rng(4)
    torch.cuda.set_device(0)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=16, device=0)
    pc = kb.PrefixCache(pool)
    base = pool.create_sequence()
    k = to_bits(kv_values(rng, (LAYERS, HKV, S, D)), BF16)
    prefill(pool, base, k, k, BF16)
    pc.store_quantized(list(range(S)), "m", base)
    hit = pc.lookup_quantized(list(range(S)), "m")
    qb = to_bits(kv_values(rng, (LAYERS, 1, HQ, D)), BF16)
    q = dev_bits(qb, BF16)
    f = hit.fork(S)
    want = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, [f], 0, q, want, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_importer, args=(q_in, q_out))
    child.start()
    try:
        q_in.put((pool.ipc_handle(), pc.describe(hit), q.cpu().view(torch.int16).numpy().tobytes()))
        tag, n = q_out.get(timeout=180)
        assert tag == "copied" and n == S
        tag, out_bytes, err = q_out.get(timeout=180)
        assert tag == "out" and err == 0
        got = np.frombuffer(out_bytes, dtype=np.float32).reshape(LAYERS, 1, HQ, D)
        np.testing.assert_array_equal(got, want.cpu().numpy())
    finally:
        child.join(timeout=60)
        if child.is_alive():
            child.terminate()
    assert child.exitcode == 0
    hit.release()
    pc.close()
    pool.close()
