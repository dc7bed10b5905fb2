"""Two-shot bf16 all-reduce over peer memory: one rank on one GPU, two ranks when the box has
two GPUs (each rank a child process, as nano-vLLM's tensor-parallel workers are).  Results are
checked bit for bit against the definition (fp32 sum in rank order, one rounding) and against
NCCL's all-reduce within bf16 rounding."""
import os

import pytest
import torch

from test_oproj_gpu import run_ranks as _run

pytestmark = pytest.mark.gpu
WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "allreduce_worker.py")


def test_single_rank(pkg):
    _run(1, WORKER)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks(pkg):
    _run(2, WORKER)


@pytest.mark.skipif(torch.cuda.device_count() < 3, reason="needs more than two GPUs")
def test_all_ranks(pkg):
    _run(torch.cuda.device_count(), WORKER)
