"""Multi-sequence serving (g4_seq_alloc / g4_forward_batch / g4_logits_batch).

Each sequence has its own KV rings; a prefill chunk of one sequence runs the
prefill kernels over that sequence's rings, and a decode step of several
sequences (one token each) runs the GEMMs over all rows and the same split
attention per row as single-sequence decode. So every batch row must give
exactly the bits of the same token decoded on a context that holds only that
sequence: logits (soft-capped) and argmax, at every step of a greedy loop,
when the batch uses the same key partition (G4_OPT_BATCH_SPLITS 148). The
default partition (fewer splits per row for large batches) changes only the
attention's summation order; its rows are checked for self-consistency.
"""
import hashlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _single(m, prompt, steps):
    for s0 in range(0, len(prompt), 512):     # chunks of <= 512 tokens, in order
        m.forward(prompt[s0:s0 + 512], s0)
    lg, am = m.logits((len(prompt) - 1) % 512)
    out = [(lg, am)]
    pos = len(prompt)
    for _ in range(steps):
        m.forward(np.array([am], np.int32), pos)
        lg, am = m.logits(0)
        out.append((lg, am))
        pos += 1
    return out


def test_batch_rows_equal_single_sequences(g4, image):
    rng = np.random.default_rng(41)
    lens = (5, 9, 3, 530)      # 530: two prefill chunks, sliding window crossed during decode
    prompts = [rng.integers(0, g4.VOCAB, size=n).astype(np.int32) for n in lens]
    steps = 3
    with g4.Model(image) as m:
        ref = [_single(m, p, steps) for p in prompts]
        m.set_option(g4.OPT_BATCH_SPLITS, 148)       # single-sequence decode's key partition
        m.seq_alloc(6, 2048)
        got = [[] for _ in prompts]
        for i, p in enumerate(prompts):           # prefill, one sequence per call, 512-token chunks
            for s0 in range(0, len(p), 512):
                m.forward_batch([i + 1], [p[s0:s0 + 512]], [s0])
            lg, am = m.logits_batch(want_logits=True)
            got[i].append((lg[0], int(am[0])))
        pos = list(lens)
        for _ in range(steps):                    # decode: all sequences in one batch
            ids = [i + 1 for i in range(len(prompts))]
            toks = [[got[i][-1][1]] for i in range(len(prompts))]
            m.forward_batch(ids, toks, pos)
            lg, am = m.logits_batch(want_logits=True)
            for i in range(len(prompts)):
                got[i].append((lg[i], int(am[i])))
            pos = [p + 1 for p in pos]
    for i in range(len(prompts)):
        for (lr, ar), (lb, ab) in zip(ref[i], got[i]):
            assert ar == ab
            assert np.array_equal(lr.view(np.uint32), lb.view(np.uint32))


def test_batch_default_splits_consistent(g4, image):
    rng = np.random.default_rng(42)
    with g4.Model(image) as m:
        m.seq_alloc(8, 1024)
        for i in range(8):
            m.forward_batch([i], [rng.integers(0, g4.VOCAB, size=20 + 7 * i).astype(np.int32)], [0])
        pos = [20 + 7 * i for i in range(8)]
        m.forward_batch(list(range(8)), [[3 + i] for i in range(8)], pos)
        lg, am = m.logits_batch(want_logits=True)
        assert np.isfinite(lg).all() and np.abs(lg).max() <= 30.0
        assert np.array_equal(am, lg.argmax(axis=1).astype(np.int32))


def test_batch_api_errors(g4, image):
    with g4.Model(image) as m:
        with pytest.raises(g4.G4Error) as e:
            m.forward_batch([0], [[1, 2]], [0])             # no sequences allocated
        assert e.value.code == -6
        m.seq_alloc(2, 64)
        with pytest.raises(g4.G4Error):
            m.forward_batch([0, 1], [[1, 2], [3]], [0, 0])  # several sequences, more than one token
        with pytest.raises(g4.G4Error):
            m.forward_batch([2], [[1]], [0])                # id beyond max_seqs
        with pytest.raises(g4.G4Error):
            m.forward_batch([0, 0], [[1], [2]], [0, 1])     # the same sequence twice
        with pytest.raises(g4.G4Error):
            m.forward_batch([0], [[1]], [1024])             # beyond the ring capacity (1024)
        with pytest.raises(g4.G4Error):
            m.forward_batch([0], [[g4.VOCAB]], [0])         # token out of range
        m.forward_batch([0, 1], [[5], [6]], [0, 0])
        _, am = m.logits_batch()
        assert am.shape == (2,)


def test_batch_step_graph_replay_equals_eager(g4, image):
    """After 32 eager steps of one row count the step is captured as a CUDA
    graph and replayed; replayed steps give the bits of eager steps
    (G4_OPT_GRAPHS 0) on the same inputs."""
    rng = np.random.default_rng(43)
    prompts = [rng.integers(0, g4.VOCAB, size=n).astype(np.int32) for n in (7, 12)]
    runs = []
    for graphs in (1, 0):
        with g4.Model(image) as m:
            m.set_option(g4.OPT_GRAPHS, graphs)
            m.seq_alloc(2, 256)
            nxt = []
            for i, p in enumerate(prompts):
                m.forward_batch([i], [p], [0])
                nxt.append(int(m.logits_batch()[1][0]))
            pos = [len(p) for p in prompts]
            out = []
            for _ in range(36):
                m.forward_batch([0, 1], [[t] for t in nxt], pos)
                lg, am = m.logits_batch(want_logits=True)
                out.append(lg.copy())
                nxt = [int(a) for a in am]
                pos = [p + 1 for p in pos]
            runs.append(out)
    for a, b in zip(*runs):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_batch_step_pdl_on_off_bitidentical(g4, image):
    """64-row decode steps (small-batch GEMMs, the transposed tcgen05 tiles
    for gate/up and the lm_head, per-row split attention; eager for 32 steps,
    then a replayed CUDA graph) give the same bits with programmatic dependent
    launch on and off: every kernel waits for its predecessor before it
    touches what the predecessor reads or writes."""
    rng = np.random.default_rng(44)
    prompts = [rng.integers(0, g4.VOCAB, size=int(n)).astype(np.int32) for n in rng.integers(5, 41, size=64)]
    runs = []
    for pdl in (1, 0):
        with g4.Model(image) as m:
            m.set_option(g4.OPT_PDL, pdl)
            m.seq_alloc(64, 256)
            nxt = []
            for i, p in enumerate(prompts):
                m.forward_batch([i], [p], [0])
                nxt.append(int(m.logits_batch()[1][0]))
            pos = [len(p) for p in prompts]
            out = []
            for _ in range(36):
                m.forward_batch(list(range(64)), [[t] for t in nxt], pos)
                lg, am = m.logits_batch(want_logits=True)
                out.append(hashlib.sha256(lg.tobytes()).hexdigest())   # 64 x 262144 logits per step
                nxt = [int(a) for a in am]
                pos = [p + 1 for p in pos]
            runs.append(out)
    assert runs[0] == runs[1]
