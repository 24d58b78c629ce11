"""Long-horizon parity of the GPU path against the CPU oracle (tests/parity_runs.py).

Two kinds of figures.  Teacher-forced runs start every step (config 1) or every layer (56
layers) from the oracle's carry / input, so each measures one kernel call's own arithmetic;
they carry the strict bars.  Free-running runs let the GPU and the oracle each carry their
own state: a requantised code that straddles a half-integer (CUDA expf / logf and FMA
contraction against numpy's unfused fp32) moves one step, persists through the decay (up
to 0.99 per step) and is amplified by the next layers, so the two trajectories drift;
their bars bound that drift.

  config 1   512 one-token codec calls on one layer's carry (the report: 2,048), all 7 layouts
             teacher-forced: >= 99.95% identical INT8/INT4 codes at every step, none more
             than one step apart, >= 99% of readouts fp16-identical
             free-running: >= 99% identical codes on average, decoded carry within 5% (L2)
             of the oracle's at every step
  56 layers  a 16-token window plus 4 decode steps, the released layouts
             teacher-forced per layer: mixer output within 1e-2 relative L2, >= 99% of the
             layer's state codes identical and >= 99.9% within one step (the multi-token bar
             of the scan tests: inside the 16-token window a code that moved at one token
             feeds the layer's later tokens, so a few codes can end several steps apart;
             measured: at most 6 steps, >= 99.86% identical in every layer); the decode
             steps' mixer outputs within 2e-2 relative L2 (each decode step starts from the
             GPU's own state after the window, which carries those code differences;
             measured 1.5e-2); the scoring head
             on the oracle's final hidden state within 1e-3 relative NLL (the north star's
             tolerance)
             free-running: window NLL within 5e-2 relative
"""
import pytest

from oracle import codec as oc
from parity_runs import config1_run, model_run

pytestmark = pytest.mark.gpu

# The tests run 512 steps per layout and mode; `python tests/parity_runs.py` writes the full
# 2,048-step report with the same code.
STEPS = 512


@pytest.mark.parametrize('layout', oc.LAYOUTS)
def test_config1_teacher_forced(layout):
    rows, s = config1_run(layout, steps=STEPS, teacher_forced=True)
    assert s['code_agreement_min'] >= 0.9995, s
    assert s['max_code_step'] <= 1, s
    assert s['y_bits_identical_mean'] >= 0.99, s


@pytest.mark.parametrize('layout', oc.LAYOUTS)
def test_config1_free_running(layout):
    rows, s = config1_run(layout, steps=STEPS, teacher_forced=False)
    assert s['code_agreement_mean'] >= 0.99, s
    assert s['carry_rel_vs_oracle_max'] <= 5e-2, s


def test_full_depth_forward_matches_oracle():
    layers, s = model_run(n_layer=56, vocab=2048, tokens=16, decode_steps=4)
    assert s['tf_mixer_rel_l2_max'] <= 1e-2, s
    assert s['tf_code_agreement_min'] >= 0.99, s
    assert s['tf_codes_within_one_min'] >= 0.999, s
    assert s['tf_decode_mixer_rel_l2_max'] <= 2e-2, s
    assert s['tf_head_nll_rel'] <= 1e-3, s
    assert s['window_nll_rel'] <= 5e-2, s
