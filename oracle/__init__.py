"""CPU oracle for the Qwen3-TTS attention + sampler + planner hot path.

TEST INFRASTRUCTURE ONLY.  These modules restate, on the CPU, the algorithms
of the reference engine (nari-labs/nari-qwen3-tts, src/nari_qwen3_tts/...)
so that the sm_100a kernels can be checked against them.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this package, and only as the checker or the timed CPU baseline;
the product path (package ``nari-qwen3-tts_b200``) never imports it and has
no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own CPU code
(its sampler, allocator and metadata builder, RMSNorm / RoPE / attention
math) on seeded inputs in a container where the reference is importable and
stores the outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks every restatement here against those fixtures.  The talker paged
attention has no CPU implementation in the reference (attend() always runs
Triton + FlashInfer); its restatement is pinned through the reference's
dense ``_depth_attention`` applied to the same KV gathered from the pages.
"""
