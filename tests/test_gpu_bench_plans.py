"""Parity at the benchmarked sizes and plans.

The other attention tests use small shapes. These run the workloads that
bench.py times — the same pool shape, sequence lengths (bench.py's own
samplers), layer count and call sequence, hence the same planner decision and
kernel instances — and check a sample of layers against the oracle:
  - configs[1] (the headline): 32 sequences, lengths U[512, 8192] from seed 1,
    Llama-3.1-8B KV shape, 32 layers;
  - configs[3] as one rank of the 8-GPU split: 2 sequences of 32,768 tokens,
    GQA 8, 48 layers, values N(0, 0.5) with 1 % outliers N(0, 8);
  - configs[4]'s sliding pool: 256 sequences with lengths U[1024, 16384]
    (seed 5), 22 layers, window 1024, max_append 256, filled 256 tokens per
    call, so every ring has wrapped several times.
Per sampled (sequence, layer): the pool's codes, scales and zeros must equal
the oracle's bit for bit, and the attention output must be within 2e-3
max-abs plus one half-ulp of the output dtype of the float64 oracle
(QuantizedKVCache.swift:71-74 + :200-204, then SDPA). Each test also asserts
the plan (krill_pool_last_plan) and the kernel instances
(krill_pool_last_kernels) that bench.py's run of the workload uses.

The unsampled layers hold device-generated N(0,1) K/V; they take part in
every launch (same plan) but are not compared.
"""
import math

import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import bench  # noqa: E402
import krill_b200 as kb  # noqa: E402
from krill_b200.shard import lpt_partition  # noqa: E402
from tests._gpu import dev_bits, host_bits  # noqa: E402

ATOL = 2e-3
TORCH_DT = {BF16: torch.bfloat16, F16: torch.float16}


def half_ulp(ref, out_dtype):
    if out_dtype == torch.float32:
        return np.zeros_like(ref)
    mant = 10 if out_dtype == torch.float16 else 7
    e = np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -14)))
    return 0.5 * 2.0 ** (e - mant)


class Workload:
    """A pool filled like bench.py fills it. Sampled layers get host-generated
    K/V (kept quantized by the oracle, per token, for the check); for a
    windowed pool only the tokens that can still be attended are host data."""

    def __init__(self, cfg, lengths, layers, sampled, window=0, outliers=False, seed=0,
                 num_blocks=None):
        self.cfg, self.layers, self.sampled, self.window = cfg, layers, list(sampled), window
        self.hq, self.hkv, self.D, self.G = cfg["hq"], cfg["hkv"], cfg["D"], cfg["G"]
        self.dt = BF16 if cfg["dtype"] == "bf16" else F16
        self.tdt = TORCH_DT[self.dt]
        self.outliers = outliers
        self.rng = np.random.default_rng(seed)
        self.gen = torch.Generator(device="cuda")
        self.gen.manual_seed(seed)
        if num_blocks is None:
            num_blocks = sum((Lq + 64 + 255) // 256 for Lq in lengths) + 8
        self.pool = kb.KVPool(layers, self.hkv, self.hq, self.D, num_blocks=num_blocks, group_size=self.G,
                              window=window, max_append=256 if window else 0)
        self.seqs = [self.pool.create_sequence() for _ in lengths]
        # (seq, sampled layer) -> list of the six quantized arrays [Hkv, S, *]
        self.q = {}
        others = [l for l in range(layers) if l not in self.sampled]
        runs = []  # contiguous runs of unsampled layers, at most 4 layers each
        for l in others:
            if runs and runs[-1][0] + runs[-1][1] == l and runs[-1][1] < 4:
                runs[-1][1] += 1
            else:
                runs.append([l, 1])
        for si, (s, Lq) in enumerate(zip(self.seqs, lengths)):
            for t0 in range(0, Lq, 256 if window else Lq):
                n = min(Lq - t0, 256 if window else Lq)
                for l0, lc in runs:
                    k = self._dev_rand((lc, 1, self.hkv, n, self.D))
                    v = self._dev_rand((lc, 1, self.hkv, n, self.D))
                    kb.append_quantize(self.pool, [s], l0, k, v)
                host = not window or t0 + n > Lq - 2 * window
                for l in self.sampled:
                    if host:
                        kbits = self._host_bits((self.hkv, n, self.D))
                        vbits = self._host_bits((self.hkv, n, self.D))
                        kb.append_quantize(self.pool, [s], l, dev_bits(kbits[None, None], self.dt),
                                           dev_bits(vbits[None, None], self.dt))
                        self._keep(si, l, kbits, vbits)
                    else:
                        k = self._dev_rand((1, 1, self.hkv, n, self.D))
                        v = self._dev_rand((1, 1, self.hkv, n, self.D))
                        kb.append_quantize(self.pool, [s], l, k, v)
        torch.cuda.synchronize()

    def _dev_rand(self, shape):
        return torch.randn(shape, generator=self.gen, device="cuda", dtype=torch.float32).to(self.tdt)

    def _host_bits(self, shape):
        return to_bits(kv_values(self.rng, shape, self.outliers), self.dt)

    def _keep(self, si, layer, kbits, vbits):
        new = list(oracle.quantize(kbits, self.dt, self.G)) + list(oracle.quantize(vbits, self.dt, self.G))
        old = self.q.get((si, layer))
        arrs = new if old is None else [np.concatenate([a, b], axis=1) for a, b in zip(old, new)]
        if self.window:  # only the last `window` rows can be attended again
            arrs = [a[:, -self.window:] for a in arrs]
        self.q[(si, layer)] = arrs

    def step(self, scale, out_dtype):
        """One decode step as bench.py runs it (krill_decode_step over every
        layer), host-generated new K/V and q; returns (q bits, output)."""
        n = len(self.seqs)
        kn = self._host_bits((self.layers, n, self.hkv, 1, self.D))
        vn = self._host_bits((self.layers, n, self.hkv, 1, self.D))
        qb = to_bits(kv_values(self.rng, (self.layers, n, self.hq, self.D)), self.dt)
        out = torch.empty((self.layers, n, self.hq, self.D), dtype=out_dtype, device="cuda")
        kb.decode_step(self.pool, self.seqs, 0, dev_bits(kn, self.dt), dev_bits(vn, self.dt),
                       dev_bits(qb, self.dt), out, scale)
        torch.cuda.synchronize()
        for (si, l) in list(self.q):
            self._keep(si, l, kn[l, si], vn[l, si])
        return qb, out.float().cpu().numpy().astype(np.float64)

    def append(self, n_new):
        """A multi-token append of host-generated K/V to every sequence."""
        n = len(self.seqs)
        kn = self._host_bits((self.layers, n, self.hkv, n_new, self.D))
        vn = self._host_bits((self.layers, n, self.hkv, n_new, self.D))
        kb.append_quantize(self.pool, self.seqs, 0, dev_bits(kn, self.dt), dev_bits(vn, self.dt))
        for (si, l) in list(self.q):
            self._keep(si, l, kn[l, si], vn[l, si])

    def check_attention(self, qb, got, scale, out_dtype, seq_ids):
        worst = 0.0
        for si in seq_ids:
            for l in self.sampled:
                ck, sk, zk, cv, sv, zv = self.q[(si, l)]
                ref = oracle.reference_attention(ck, sk, zk, cv, sv, zv, qb[l, si], self.dt, self.G, scale)
                err = np.abs(got[l, si] - ref)
                assert np.all(err <= ATOL + half_ulp(ref, out_dtype)), (
                    f"seq {si} layer {l}: max err {err.max():.3e}")
                worst = max(worst, float(err.max()))
        return worst

    def check_codes(self, seq_ids):
        """The pool's stored codes, scales and zeros equal the oracle's."""
        for si in seq_ids:
            for l in self.sampled:
                snap = self.seqs[si].quantized_snapshot(l)
                mine = [snap.keys, snap.key_scales, snap.key_zeros, snap.values, snap.value_scales,
                        snap.value_zeros]
                for name, a, want in zip(("codes K", "scale K", "zero K", "codes V", "scale V", "zero V"),
                                         mine, self.q[(si, l)]):
                    a = a.cpu().numpy() if a.dtype == torch.uint8 else host_bits(a)
                    a = a[:, -want.shape[1]:]
                    assert np.array_equal(a, want), f"seq {si} layer {l}: {name} differ from the oracle"


from tests._bench_plans import PLANS  # noqa: E402


def _assert_plan(pool, key):
    plan, kernels = PLANS[key]
    assert pool.last_plan() == plan, f"{key}: plan {pool.last_plan()} != bench's {plan}"
    assert pool.last_kernels() == kernels, f"{key}: kernels {pool.last_kernels()} != {kernels}"


def test_headline_batch32_plan_and_parity():
    cfg = bench.CONFIGS["llama31_8b_batch32"]
    lengths_all = bench.sample_lengths(cfg, cfg["seqs"])
    lengths = [lengths_all[i] for i in lpt_partition(lengths_all, 1)[0]]
    w = Workload(cfg, lengths, cfg["layers"], sampled=[0, 17, 31], seed=101)
    w.check_codes(range(len(lengths)))
    for _ in range(2):
        qb, got = w.step(cfg["scale"], torch.bfloat16)
        _assert_plan(w.pool, "llama31_8b_batch32")
        w.check_attention(qb, got, cfg["scale"], torch.bfloat16, range(len(lengths)))
    w.check_codes(range(len(lengths)))
    assert w.pool.device_error() == 0
    w.pool.close()


def test_longctx_gqa8_outliers_rank_of_8gpu_plan_and_parity():
    cfg = bench.CONFIGS["qwen3_30b_longctx"]
    lengths = bench.sample_lengths(cfg, 2)
    w = Workload(cfg, lengths, cfg["layers"], sampled=[0, 47], outliers=True, seed=103)
    w.check_codes(range(2))
    for _ in range(2):
        qb, got = w.step(cfg["scale"], torch.bfloat16)
        _assert_plan(w.pool, "qwen3_30b_longctx/8gpu")
        w.check_attention(qb, got, cfg["scale"], torch.bfloat16, range(2))
    w.check_codes(range(2))
    assert w.pool.device_error() == 0
    w.pool.close()


def test_mixed_sliding_pool_plan_and_parity():
    cfg = bench.CONFIGS["gemma_mixed_256"]
    lengths = bench.sample_lengths(cfg, cfg["seqs"])
    W = cfg["window"]
    w = Workload(cfg, lengths, cfg["layers_sliding"], sampled=[0, 21], window=W, seed=105,
                 num_blocks=cfg["seqs"] * 5 + 8)
    for s, Lq in zip(w.seqs, lengths):
        assert s.length(0) == Lq
    sample = list(range(0, cfg["seqs"], 5))
    w.check_codes(sample)
    for _ in range(2):
        qb, got = w.step(cfg["scale"], torch.float16)
        _assert_plan(w.pool, "gemma_mixed_256/sliding")
        w.check_attention(qb, got, cfg["scale"], torch.float16, sample)
    w.check_codes(sample)
    assert w.pool.device_error() == 0
    w.pool.close()


def test_sliding_ring_wraps_across_multi_and_single_token_appends():
    """configs[4]'s sliding layers (window 1024, max_append 256, head_dim 256,
    GQA 2, scale 1) on lengths that wrap the 5-block ring several times, with
    multi-token appends between single-token decode steps
    (RotatingKVCache.swift:71-113: retain window - 1 rows, then append; the
    attention sees the last `window` tokens). Every layer is compared."""
    cfg = dict(bench.CONFIGS["gemma_mixed_256"])
    W = cfg["window"]
    w = Workload(cfg, [1100, 2500, 5000], 2, sampled=[0, 1], window=W, seed=107)
    for op in ["step", 100, "step", "step", 256, "step", 37, 255, "step"]:
        if op == "step":
            qb, got = w.step(cfg["scale"], torch.float32)
            w.check_attention(qb, got, cfg["scale"], torch.float32, range(3))
        else:
            w.append(op)
    w.check_codes(range(3))
    assert w.pool.device_error() == 0
    w.pool.close()
