"""CPU oracle for the SQ3.25 / FP4-G16 Mamba-2 hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use it, and
there only as the checker or the timed CPU baseline, never as the product.

Contents:
  codec.py   numpy restatement of the production latent codec kernel
             (scripts/fp4_zero_predictor_codec_v1.py:76-181), its host-side
             predictor correction (:221-225), the requantizer
             (scripts/state_ppl_codec_v6.py:52-61), the layout chain
             (scripts/w4_state_repair_codec_v2.py:22-45) and FP8-E4M3 byte
             arithmetic.
  fp4.py     numpy restatement of E2M1 / E4M3 G16 weight decode and encode
             (mamba2_recall/fp4.py:85-154, 157-219, 259-269).
  model.py   torch-CPU restatement of one Mamba-2 layer, the Resurface adapter
             and the scoring / greedy loops that call the codec.

Pinning: codec.py and fp4.py are checked bit-for-bit against golden vectors
produced by running the reference's own code in the build container
(tests/golden/make_golden.py). The mamba_ssm pieces in model.py (RMSNorm,
gated RMSNorm, Block residual, conv prefill) have no runnable reference here;
their parity is UNPINNED and follows the public Mamba-2 definition.
"""
