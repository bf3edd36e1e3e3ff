"""The decode-attention plan and kernel instances of each bench.py workload,
as (piece sub-blocks, kv heads per item, items, CTAs) and the '+'-joined
instance names of krill_pool_last_kernels. Pinned on the CPU by dry-run pools
over every step bench.py times (tests/test_bench_plans.py) and on the GPU by
tests/test_gpu_bench_plans.py; bench.py prints the same two values in its
JSON line."""

PLANS = {
    # configs[1], the headline: 32 sequences, lengths U[512, 8192] (seed 1)
    "llama31_8b_batch32": ((64, 8, 1536, 148), "attn_tc_kernel<128,2,8,1,13,0>+attn_combine_kernel<128>"),
    # configs[3] on one GPU (16 x 32,768 tokens) and per rank at 8 GPUs (2 each)
    "qwen3_30b_longctx": ((128, 4, 3840, 148), "attn_tc_kernel<128,2,8,2,12,0>+attn_combine_kernel<128>"),
    "qwen3_30b_longctx/8gpu": ((64, 4, 864, 148), "attn_tc_kernel<128,2,8,2,12,0>+attn_combine_kernel<128>"),
    # configs[4]'s 22 sliding layers: 256 sequences, window 1024
    "gemma_mixed_256/sliding": ((128, 4, 5632, 148), "attn_tc_kernel<256,4,8,2,11,0>"),
}
