"""bench.engine_watchdog (CPU): a worker process that dies ends the run within seconds
instead of leaving rank 0 waiting in a collective."""
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import multiprocessing as mp, sys, time
sys.path.insert(0, {root!r})
import bench

def worker(code, linger=0.5):
    time.sleep(linger)
    sys.exit(code)

def other(code):
    time.sleep(0.3)
    sys.exit(code)

if __name__ == "__main__":
    ctx = mp.get_context("spawn")
    stop = bench.engine_watchdog(worker, period=0.1)
    ok = ctx.Process(target=worker, args=(0,), kwargs={{"linger": 60}})
    ok.start()
    ctx.Process(target=worker, args=({code},)).start()
    ctx.Process(target=other, args=(5,)).start()   # not a worker: its exit code is ignored
    time.sleep(8)    # stands for rank 0 blocked in a collective
    stop.set()       # the measured work is done; shutdown may end workers any way
    ok.kill()
    time.sleep(0.5)
    print("not stopped")
"""


def run(tmp_path, code):
    script = tmp_path / "rank0.py"  # a file: spawned children import their target from it
    script.write_text(SCRIPT.format(root=ROOT, code=code))
    t0 = time.time()
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=120)
    return r, time.time() - t0


def test_dead_worker_stops_the_run(tmp_path):
    r, dt = run(tmp_path, 7)
    assert r.returncode == 3, r.stdout + r.stderr
    assert '"error"' in r.stdout and "exited with code 7" in r.stdout
    assert dt < 20


def test_clean_exit_is_not_an_error(tmp_path):
    r, dt = run(tmp_path, 0)
    assert r.returncode == 0 and "not stopped" in r.stdout, r.stdout + r.stderr
