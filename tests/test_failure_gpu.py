"""Failure detection on the GPU without a GPU fault.

Every wait in the persistent decode kernel is bounded (2 s of %globaltimer):
a consumer whose weight stage never lands gives up, records a timeout in the
context's device error word, leaves its loops as whole warps and returns; the
CTAs behind it give up at the next grid barrier the same way. This test makes
those waits run out on purpose with the test aid g4_test_starve_next_step (the
next step's weight producers issue no copies: a flag that nothing sets), and
checks that
  - the step reports G4_ERR_DEVICE with a wait-timeout message at the next
    synchronising call (g4_logits), and the process and context stay usable;
  - the context recovers (error word and barrier counters reset): the same
    step run again gives logits and argmax bit-identical to a context that
    never failed.
No kernel traps or hangs: the failure is a status the host reads.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_starved_step_times_out_and_context_recovers(g4, image):
    rng = np.random.default_rng(31)
    toks = rng.integers(0, g4.VOCAB, size=9).astype(np.int32)
    with g4.Model(image) as good:
        good.forward(toks[:8], 0)
        good.forward(toks[8:9], 8)
        want, want_am = good.logits(0)
    with g4.Model(image) as m:
        m.forward(toks[:8], 0)
        g4._check(m.L.g4_test_starve_next_step(m.h), m.h)
        m.forward(toks[8:9], 8)
        with pytest.raises(g4.G4Error) as ei:
            m.logits(0)
        assert ei.value.code == -5                      # G4_ERR_DEVICE
        assert "timed out" in str(ei.value)
        m.sync()                                        # nothing left pending, no error
        # the same step again, now with its weights streamed
        m.forward(toks[8:9], 8)
        got, got_am = m.logits(0)
        assert got_am == want_am
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
