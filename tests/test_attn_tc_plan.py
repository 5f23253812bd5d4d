"""The tensor-core prefill attention's schedule, checked on the host (CPU, no
GPU work): g4k_attn_tc_plan rebuilds the plan the launches use for a chunk of
T tokens at start_pos on a GPU with a given SM count and verifies that the S
tiles lie inside the workspace and hold every row's visible keys, that the
P V K-stages of every (row tile, dimension tile) pair are covered exactly once
by the per-CTA runs, that the partial slots are distinct, and that the
combine's CTA range of every pair is exactly the CTAs that ran it.
"""
import numpy as np
import pytest


CASES = [
    (512, 512, 0, 148), (512, 512, 15872, 148), (512, 512, 131072 - 512, 148), (512, 1, 0, 148),
    (512, 17, 1000, 148), (512, 96, 0, 1), (512, 512, 4000, 7), (512, 64, 4000, 132),
    (256, 512, 0, 148), (256, 512, 1536, 148), (256, 300, 700, 148), (256, 64, 3000, 132),
    (256, 1, 511, 148), (256, 512, 131072 - 512, 148), (256, 33, 510, 5),
]


@pytest.mark.parametrize("hd,T,start_pos,sms", CASES)
def test_schedule_covers_every_stage_once(g4, hd, T, start_pos, sms):
    rc, units_s, stages_o, ctas_o, ws = g4.attn_tc_plan(hd, T, start_pos, sms)
    assert rc == 0, f"schedule check {rc} failed"
    assert units_s >= 1 and stages_o >= 1 and 1 <= ctas_o <= stages_o and ws > 0
    # short chunks: one CTA per (row tile, dimension tile) pair; long ones: one run per SM
    pairs = (8 * T + 127) // 128 * (hd // 256)
    assert ctas_o == pairs if stages_o <= 24 * pairs else ctas_o == min(sms, stages_o)


def test_schedule_random_chunks(g4):
    rng = np.random.default_rng(5)
    for _ in range(200):
        hd = int(rng.choice([256, 512]))
        T = int(rng.integers(1, 513))
        sp = int(rng.integers(0, 131072 - T + 1)) if rng.random() < 0.3 else int(rng.integers(0, 4096))
        sms = int(rng.choice([1, 3, 64, 132, 148]))
        rc = g4.attn_tc_plan(hd, T, sp, sms)[0]
        assert rc == 0, (hd, T, sp, sms, rc)


def test_schedule_rejects_bad_chunks(g4):
    assert g4.attn_tc_plan(384, 16, 0)[0] != 0          # head dimension
    assert g4.attn_tc_plan(512, 513, 0)[0] != 0         # more than one chunk
    assert g4.attn_tc_plan(512, 16, 131072 - 8)[0] != 0  # past the context
