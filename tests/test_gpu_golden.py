"""The CUDA kernels against the committed golden fixtures (tests/golden/):
quantize+append bit-exact (codes, scales, zeros, dequantized fp16), decode
attention within 2e-3 max-abs of the float64 reference values."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, host_bits  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(prefix):
    files = sorted(f for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".npz"))
    assert files
    return [(f, np.load(os.path.join(GOLDEN, f))) for f in files]


def test_golden_quantize():
    for name, z in _load("quant_"):
        x = z["x"]
        rows, D = x.shape
        G, dt, var = int(z["G"]), int(z["dtype"]), int(z["variant"])
        # rows become tokens of one (layer, head); K and V get the same rows
        pool = kb.KVPool(1, 1, 1, D, num_blocks=4, group_size=G, quant_variant=var)
        s = pool.create_sequence()
        t = dev_bits(np.ascontiguousarray(x[None, None, None]), dt)
        kb.append_quantize(pool, [s], 0, t, t)
        snap = s.quantized_snapshot(0)
        kd, vd = s.snapshot(0)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(snap.keys.cpu().numpy()[0], z["codes"], err_msg=name)
        np.testing.assert_array_equal(snap.values.cpu().numpy()[0], z["codes"], err_msg=name)
        np.testing.assert_array_equal(host_bits(snap.key_scales)[0], z["scales"], err_msg=name)
        np.testing.assert_array_equal(host_bits(snap.key_zeros)[0], z["zeros"], err_msg=name)
        np.testing.assert_array_equal(host_bits(kd)[0], z["deq"], err_msg=name)
        np.testing.assert_array_equal(host_bits(vd)[0], z["deq"], err_msg=name)
        pool.close()


def test_golden_attention():
    for name, z in _load("attn_"):
        k, v, q = z["k"], z["v"], z["q"]
        hkv, L, D = k.shape
        hq, G, dt = int(z["hq"]), int(z["G"]), int(z["dtype"])
        pool = kb.KVPool(1, hkv, hq, D, num_blocks=4, group_size=G)
        s = pool.create_sequence()
        kb.append_quantize(pool, [s], 0, dev_bits(np.ascontiguousarray(k[None, None]), dt),
                           dev_bits(np.ascontiguousarray(v[None, None]), dt))
        out = torch.empty((1, 1, hq, D), dtype=torch.float32, device="cuda")
        kb.decode_attention(pool, [s], 0, dev_bits(np.ascontiguousarray(q[None, None]), dt), out,
                            float(z["scale"]))
        torch.cuda.synchronize()
        err = np.abs(out.cpu().numpy()[0, 0].astype(np.float64) - z["out"]).max()
        assert err <= 2e-3, f"{name}: {err:.3e}"
        pool.close()
