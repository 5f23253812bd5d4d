"""The C host (gemma4.c_b200/host/run.c) on the GPU: gemma4.c's command line
over libg4cuda.so. `--bench P G` prints the reference's ppP / tgG@dP lines
(gemma4.c:627-645); `--dump-logits` writes every prompt position's logits
(gemma4.c:563-572), which must equal the library's g4_logits_rows for the same
token ids bit for bit; greedy generation (-t 0) runs to -n tokens."""
import os
import re
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gemma4.c_b200")


@pytest.fixture(scope="module")
def model_file(g4):
    d = tempfile.mkdtemp(prefix="g4host")
    path = os.path.join(d, "synth.bin")
    g4._check(g4.load().g4synth_write_file(path.encode(), 0, 0))
    yield path
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture(scope="module")
def run_exe():
    exe = os.path.join(PKG, "run")
    if not os.path.exists(exe):
        subprocess.run(["make", "-C", PKG, "run"], check=True, capture_output=True)
    return exe


def test_bench_lines(run_exe, model_file):
    r = subprocess.run([run_exe, "-m", model_file, "--bench", "512", "8"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    pp = re.search(r"^pp512 ([0-9.]+) tok/s$", r.stdout, re.M)
    tg = re.search(r"^tg8@d512 ([0-9.]+) tok/s$", r.stdout, re.M)
    assert pp and tg, r.stdout
    print(r.stdout)
    assert float(pp.group(1)) > 0 and float(tg.group(1)) > 0


def test_dump_logits_equal_library(g4, run_exe, model_file):
    prompt = "Hello, B200 world"
    r = subprocess.run([run_exe, "-m", model_file, "--dump-logits", prompt], capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr
    # the synthetic model's tokenizer section is zero: <bos> then byte tokens, spaces as U+2581
    ids = np.array([2] + [238 + b for b in prompt.replace(" ", "▁").encode()], np.int32)
    got = np.frombuffer(r.stdout, np.float32).reshape(-1, g4.VOCAB)
    assert got.shape[0] == ids.size
    img = g4.synth_image(seed=0, flags=0)
    with g4.Model(img) as m:
        m.forward(ids, 0)
        want = m.logits_rows(0, ids.size)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_greedy_generation_runs(run_exe, model_file):
    r = subprocess.run([run_exe, "-m", model_file, "-t", "0", "-n", "8", "Why is the sky blue?"],
                       capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr
