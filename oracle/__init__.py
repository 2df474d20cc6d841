"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in fp32 PyTorch on the CPU, the reference engine's own attention arithmetic (the fp32 paths that
saicherry93479/Qwen3-TTS-Engine itself uses as its parity oracle: engine/talker.py:82-88, engine/talker.py:163-167,
engine/arrivals.py:125-131, engine/code_predictor.py:46-47) plus the frame step around it. It is the checker, never the
thing measured or shipped: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
it. The product path (the q3attn package) never imports it and fails loudly when its CUDA library is missing.

Parity is pinned: tests/golden/make_golden.py imports the reference's own modules (engine.talker, engine.arrivals,
engine.code_predictor) in the build container, runs them on seeded inputs and commits their outputs as fixtures; the
CPU tests check this restatement against those fixtures.
"""
