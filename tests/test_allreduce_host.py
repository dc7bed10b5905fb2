"""Host-side checks of allreduce.AllReduce without a GPU: which tensors it accepts and the
arguments it passes to b200_allreduce_bf16 (the kernel itself: tests/test_allreduce_gpu.py)."""
import pytest
import torch


class _Lib:
    def __init__(self):
        self.calls = []

    def b200_allreduce_bf16(self, *args):
        self.calls.append(args)
        return 0


def _op(monkeypatch, pkg, max_elems=64):
    from learn_nano_vllm_b200 import allreduce
    fake = _Lib()
    monkeypatch.setattr(allreduce, "lib", lambda: fake)
    monkeypatch.setattr(allreduce.torch.cuda, "current_stream", lambda dev=None: type("S", (), {"cuda_stream": 0})())
    op = allreduce.AllReduce.__new__(allreduce.AllReduce)
    op.max_elems, op.buf_elems, op.rank, op.world = max_elems, 2 * max_elems, 1, 2
    op.bufs = torch.zeros(2 * max_elems, dtype=torch.bfloat16)
    op.buf_ptrs = torch.zeros(2, dtype=torch.int64)
    op.flag_ptrs = torch.zeros(2, dtype=torch.int64)
    return op, fake


def test_slots_and_plain_tensors_are_accepted(monkeypatch, pkg):
    op, fake = _op(monkeypatch, pkg)
    x = torch.zeros(32, dtype=torch.bfloat16)
    assert op(x) is x                                  # in place
    y = torch.empty_like(x)
    assert op(x, out=y) is y
    xi, yo = op.input_buffer(32), op.result_buffer(32)
    assert op(xi, out=yo) is yo                        # zero-copy slots
    assert op(op.result_buffer(32), out=op.input_buffer(32)).data_ptr() == op.bufs.data_ptr()
    out_ptr, in_ptr, n, bufs, buf_elems, flags, rank, world, stream = fake.calls[2]
    assert (out_ptr, in_ptr, n, buf_elems, rank, world) == (yo.data_ptr(), xi.data_ptr(), 32, 128, 1, 2)


def test_views_inside_the_slots_are_refused(monkeypatch, pkg):
    op, fake = _op(monkeypatch, pkg)
    with pytest.raises(AssertionError, match="slot buffer"):
        op(op.bufs[8:40])
    with pytest.raises(AssertionError, match="slot buffer"):
        op(torch.zeros(32, dtype=torch.bfloat16), out=op.bufs[70:102])
    with pytest.raises(AssertionError):
        op(torch.zeros(65, dtype=torch.bfloat16))      # above max_elems
    assert fake.calls == []
