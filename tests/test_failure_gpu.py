"""Failure detection on the GPU without a fault: every device-side wait of the engine is bounded,
and a wait that runs out ends the step early, records FENCE_E_DEVICE_WAIT (-5) in the device error
word and surfaces on the host as an error status, with the context still usable.

The test makes one wait run out on purpose: fence_load_opts.wait_test_phase gives the grid-counter
wait of one step-kernel phase a target that no CTA ever reaches (a flag that nothing sets), so each
CTA's bounded poll (about a second) expires. Nothing faults, traps or hangs."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("phase", [1, 3])  # the first attention phase; the first gate/up phase
def test_step_wait_runs_out_and_reports(fb, orc, tmp_path, phase):
    import torch
    assert torch.cuda.is_available()
    p = str(tmp_path / "tiny.gguf")
    fb.synth_write(p, "tiny-q6k", seed=41)
    fb.lib().fence_device_error()  # start from a clear word
    m = fb.Model(p, max_ctx=64, wait_test_phase=phase)
    with pytest.raises(fb.FenceError) as err:
        m.forward(3, 0)
    assert "bounded wait expired" in str(err.value)
    assert fb.lib().fence_device_error() == -5  # read and cleared
    m.close()
    # the GPU still answers: a model without the test option decodes and matches the oracle
    m = fb.Model(p, max_ctx=64)
    ora = orc.OracleModel(p, max_ctx=64, kv_bf16=False, threads=4)
    worst = 0.0
    for pos, tok in enumerate([3, 141, 59]):
        m.forward(tok, pos)
        worst = max(worst, float(np.max(np.abs(m.logits() - ora.forward(tok, pos)))))
    m.close()
    ora.close()
    assert worst < 2e-3, worst
    assert fb.lib().fence_device_error() == 0


def test_decode_greedy_reports_expired_wait(fb, tmp_path):
    """The device-resident decode loop (no host round trip per token) reports the expired wait of
    any of its steps once it synchronises."""
    p = str(tmp_path / "tiny.gguf")
    fb.synth_write(p, "tiny-q8", seed=43)
    fb.lib().fence_device_error()
    m = fb.Model(p, max_ctx=64, wait_test_phase=4)
    with pytest.raises(fb.FenceError) as err:
        m.decode_greedy(5, 0, 3)
    assert "bounded wait expired" in str(err.value)
    assert fb.lib().fence_device_error() == -5
    m.close()
