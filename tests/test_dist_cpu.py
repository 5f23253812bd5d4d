"""bench.py's multi-rank plumbing on CPU: two ranks over gloo (127.0.0.1).

`bench.py --gpus N` under torchrun runs one model replica per GPU; the process
group only provides the barrier around the timed region and the max over ranks
of the device times. Here the same Dist class runs as two CPU processes.
"""
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import sys
sys.path.insert(0, {root!r})
import bench
d = bench.Dist()
assert d.world == 2 and d.pg
v = d.max(10.0 * d.rank + 1.0)        # rank 1 has the larger time
d.barrier()
print("MAX", d.rank, v, flush=True)
d.close()
"""

SCRIPT_REF = r"""
import sys
sys.path.insert(0, {root!r})
import bench
class A: pass
d = bench.Dist.__new__(bench.Dist)
d.rank, d.world, d.local, d.pg = 1, 2, 0, None
bench.run_reference_arm(A(), d)       # a rank other than 0 returns at once
print("REF-RANK1-OK", flush=True)
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_barrier_and_max():
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, "-c", SCRIPT.format(root=ROOT)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=240) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, e[-2000:]
    got = sorted(line.split()[1:] for o, _ in outs for line in o.splitlines() if line.startswith("MAX"))
    assert got == [["0", "11.0"], ["1", "11.0"]]


def test_reference_arm_other_ranks_exit():
    r = subprocess.run([sys.executable, "-c", SCRIPT_REF.format(root=ROOT)], capture_output=True, text=True,
                       timeout=120, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-2000:]
    assert "REF-RANK1-OK" in r.stdout
