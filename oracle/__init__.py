"""CPU oracle for the MOSS-TTS batch-1 decode hot path.

TEST INFRASTRUCTURE ONLY. This package is a plain numpy restatement of the
reference implementation's arithmetic (kadirnar/MOSS-TTS-optimized,
``src/moss_tts``), used as the checker for the CUDA path. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it; the product package never does, and the product
path fails loudly when its CUDA library is missing.

Pinning: every function here is checked against golden vectors produced by the
reference's own CPU-runnable code (``calibrated_backend.unpack_signed``,
``calibrated_quant.dequantize``, ``dp4a_packing.pack_interleaved``,
``torch.nn.functional.linear`` and the upstream HF ``Qwen3`` / ``MossTTSDelayModel``
modules), written by ``tests/golden/make_golden.py`` and checked by
``tests/test_oracle_golden.py``.

Modules:
  numerics  bf16 round-to-nearest-even helpers (numpy has no bfloat16)
  quant     int4/G32 weight formats and dequantization
  ops       RMSNorm, QK-norm + RoPE, split-K attention, SiLU, embedding, heads
  model     one full decode step of the MOSS-TTS backbone
"""
