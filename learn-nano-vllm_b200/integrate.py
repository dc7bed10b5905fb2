"""Install the B200 attention path into an unmodified nano-vLLM.

nano-vLLM constructs `Attention` inside Qwen3Attention (nanovllm/models/qwen3.py:61-66),
which imported the class by name (qwen3.py:7).  install() rebinds that name
(and the one in nanovllm.layers.attention) to this package's module, and
points it at the reference's own context (nanovllm/utils/context.py), so that
ModelRunner, BlockManager, the prefix cache, the scheduler and CUDA-graph
capture run unchanged on top of the B200 kernels.  Call it before the engine
builds its model.
"""
import importlib

import torch

from . import attention as _attention
from .ops import store_kvcache


def _fused_qwen3_attention_forward(self, positions, hidden_states):
    """Qwen3Attention.forward (nanovllm/models/qwen3.py:72-88) with q/k norm, RoPE and the
    KV-cache store fused into one kernel (Attention.forward_fused)."""
    if (self.qkv_bias or self.head_dim != 128 or not isinstance(self.attn, _attention.Attention)
            or hidden_states.dtype not in (torch.bfloat16, torch.float16)):
        return _ORIGINAL_FORWARD[0](self, positions, hidden_states)
    qkv = self.qkv_proj(hidden_states)
    o = self.attn.forward_fused(qkv, positions, self.q_norm, self.k_norm, self.rotary_emb)
    return self.o_proj(o.flatten(1, -1))


_ORIGINAL_FORWARD = []
_ORIGINAL_SAMPLER = []
_ORIGINAL_PREPARE = []


def _device_prepare_decode(self, seqs):
    """ModelRunner.prepare_decode (nanovllm/engine/model_runner.py:167-187) with the metadata
    expanded on the device from one packed copy (decode_meta.DecodeMetadata)."""
    from nanovllm.utils.context import set_context
    from .decode_meta import DecodeMetadata
    meta = self.__dict__.get("_b200_meta")
    if meta is None:
        meta = self._b200_meta = DecodeMetadata()
    # worker ranks get trimmed sequences without temperatures and do not sample
    input_ids, positions, slot_mapping, context_lens, block_tables, temps = meta.build(
        seqs, self.block_size, temperatures=self.rank == 0)
    set_context(False, slot_mapping=slot_mapping, context_lens=context_lens, block_tables=block_tables)
    self._b200_temps = (seqs, temps)
    return input_ids, positions


def _device_prepare_sample(self, seqs):
    """ModelRunner.prepare_sample (model_runner.py:189-193): the temperatures of a decode batch
    come with its device metadata; other batches use the reference's code."""
    cached = self.__dict__.get("_b200_temps")
    if cached is not None and cached[0] is seqs:
        return cached[1]
    return _ORIGINAL_PREPARE[1](self, seqs)


class _RowParallelState:
    """The fused GEMM + all-reduce buffers of this process, one per (output size, device),
    shared by every RowParallelLinear (they run one after another on one stream)."""
    ops = {}
    # Decode-sized batches only (nano-vLLM captures decode graphs up to 512 sequences): there the
    # fused kernel beats F.linear + NCCL (1.15-1.6x at TP2); prefill batches of thousands of rows
    # run its GEMM below cuBLAS, so they take the stock path.
    max_tokens = 512

    @classmethod
    def get(cls, n, device):
        key = (n, device)
        op = cls.ops.get(key)
        if op is None:
            import torch.distributed as dist
            from .oproj import OprojAllReduce
            op = cls.ops[key] = OprojAllReduce(dist.group.WORLD, max_tokens=cls.max_tokens, hidden=n, device=device)
        return op


_ORIGINAL_ROW = []


def _fused_row_parallel_forward(self, x):
    """RowParallelLinear.forward (nanovllm/layers/linear.py:152-156): this rank's F.linear and
    the all-reduce over the tensor-parallel ranks as one kernel (oproj.OprojAllReduce), for
    bias-free bf16 layers with N % 256 == 0 and K % 64 == 0 and activations the kernel's tensor
    maps can address (unit inner stride, 16-byte aligned rows).  Every rank sees the same batch
    and the same layer shapes, so every rank takes the same branch (the kernel is collective)."""
    n, k = self.weight.shape
    if (self.tp_size == 1 or self.bias is not None or x.dtype != torch.bfloat16 or x.dim() != 2
            or n % 256 or k % 64 or x.shape[0] > _RowParallelState.max_tokens or x.stride(-1) != 1
            or x.stride(0) % 8 or x.data_ptr() % 16):
        return _ORIGINAL_ROW[0](self, x)
    return _RowParallelState.get(n, x.device)(x, self.weight)


class _AllReduceState:
    """The two-shot all-reduce buffers of this process, one per (row width, device), shared by
    every RowParallelLinear (they run one after another on one stream)."""
    ops = {}
    # Decode-sized outputs only (nano-vLLM captures decode graphs up to 512 sequences); prefill
    # batches keep NCCL.  The buffers are made by the eager decode forward that precedes each
    # graph capture (model_runner.py:236-246), never during a capture.
    max_tokens = 512

    @classmethod
    def get(cls, n, device):
        key = (n, device)
        op = cls.ops.get(key)
        if op is None:
            import torch.distributed as dist
            from .allreduce import AllReduce
            op = cls.ops[key] = AllReduce(dist.group.WORLD, cls.max_tokens * n, device=device)
        return op


def _allreduce_row_parallel_forward(self, x):
    """RowParallelLinear.forward (nanovllm/layers/linear.py:152-156) with the reference's F.linear
    and, for contiguous 16-byte aligned bf16 outputs of at most max_tokens rows, this package's
    two-shot all-reduce over peer memory (allreduce.AllReduce) in place of dist.all_reduce.  Every
    rank sees the same batch and layer shapes, so every rank takes the same branch."""
    import torch.distributed as dist
    y = torch.nn.functional.linear(x, self.weight, self.bias if self.tp_rank == 0 else None)
    if self.tp_size > 1:
        rows = y.numel() // y.shape[-1] if y.dim() else 0
        if (y.dtype == torch.bfloat16 and y.dim() >= 1 and y.is_contiguous() and 0 < rows <= _AllReduceState.max_tokens
                and y.numel() % 8 == 0 and y.data_ptr() % 16 == 0):
            _AllReduceState.get(y.shape[-1], y.device)(y.view(-1))
        else:
            dist.all_reduce(y)
    return y


class _FusedSamplerState:
    """Seed and per-call offset of the fused sampler's counter-based noise."""
    seed = 0
    offset = 0


def _fused_sampler_forward(self, logits, temperatures):
    """Sampler.forward (nanovllm/layers/sampler.py:7-12) as one fused kernel: the same
    exponential race, with its Exp(1) noise drawn in-kernel (fresh offset per call)."""
    from .ops import sample
    _FusedSamplerState.offset += 1
    return sample(logits, temperatures, seed=_FusedSamplerState.seed, offset=_FusedSamplerState.offset)


def install(fuse_qk_epilogue: bool = False, fuse_sampler: bool = False, workers: bool = False,
            worker_setup: tuple = (), device_metadata: bool = False, fuse_row_parallel: bool = False,
            row_parallel_allreduce: bool = False):
    """Patch the importable `nanovllm` package; returns the patched modules.

    With fuse_qk_epilogue, Qwen3Attention.forward also runs q/k RMSNorm, RoPE and
    the KV-cache store as one kernel (ops.qk_norm_rope_store) instead of the
    reference's separate RMSNorm / RotaryEmbedding modules and store.  With
    fuse_sampler, Sampler.forward becomes the one-pass fused sampler (ops.sample;
    its noise stream is seeded from torch.initial_seed()).  With device_metadata,
    ModelRunner.prepare_decode / prepare_sample build the decode step's tensors on
    the device from one packed host-to-device copy (decode_meta).  With
    fuse_row_parallel, RowParallelLinear.forward (o_proj, down_proj) runs its GEMM and
    the tensor-parallel all-reduce as one kernel over peer memory (oproj); every rank must run
    it, so it implies workers.  With row_parallel_allreduce (and not fuse_row_parallel),
    RowParallelLinear.forward keeps F.linear and replaces its NCCL all-reduce with this
    package's two-shot all-reduce (allreduce.AllReduce) for decode-sized outputs; it too implies
    workers.  With workers, the
    engine's tensor-parallel ranks (spawned processes, nanovllm/engine/llm_engine.py:24-30)
    run install() with the same options before building their ModelRunner;
    worker_setup lists "module:function" hooks they run first.
    """
    ctx_mod = importlib.import_module("nanovllm.utils.context")
    attn_mod = importlib.import_module("nanovllm.layers.attention")
    qwen3 = importlib.import_module("nanovllm.models.qwen3")
    _attention.set_context_source(ctx_mod.get_context)
    attn_mod.Attention = _attention.Attention
    attn_mod.store_kvcache = store_kvcache
    qwen3.Attention = _attention.Attention
    if not _ORIGINAL_FORWARD:
        _ORIGINAL_FORWARD.append(qwen3.Qwen3Attention.forward)
    qwen3.Qwen3Attention.forward = _fused_qwen3_attention_forward if fuse_qk_epilogue else _ORIGINAL_FORWARD[0]
    sampler_mod = importlib.import_module("nanovllm.layers.sampler")
    if not _ORIGINAL_SAMPLER:
        _ORIGINAL_SAMPLER.append(sampler_mod.Sampler.forward)
    if fuse_sampler:
        _FusedSamplerState.seed = torch.initial_seed() & (2 ** 64 - 1)
    sampler_mod.Sampler.forward = _fused_sampler_forward if fuse_sampler else _ORIGINAL_SAMPLER[0]
    engine_mod = importlib.import_module("nanovllm.engine.llm_engine")
    runner_mod = importlib.import_module("nanovllm.engine.model_runner")
    if not _ORIGINAL_PREPARE:
        _ORIGINAL_PREPARE.extend([runner_mod.ModelRunner.prepare_decode, runner_mod.ModelRunner.prepare_sample])
    runner_mod.ModelRunner.prepare_decode = _device_prepare_decode if device_metadata else _ORIGINAL_PREPARE[0]
    runner_mod.ModelRunner.prepare_sample = _device_prepare_sample if device_metadata else _ORIGINAL_PREPARE[1]
    linear_mod = importlib.import_module("nanovllm.layers.linear")
    if not _ORIGINAL_ROW:
        _ORIGINAL_ROW.append(linear_mod.RowParallelLinear.forward)
    linear_mod.RowParallelLinear.forward = (_fused_row_parallel_forward if fuse_row_parallel else
                                            _allreduce_row_parallel_forward if row_parallel_allreduce else
                                            _ORIGINAL_ROW[0])
    if workers or fuse_row_parallel or row_parallel_allreduce:
        import functools
        entry = importlib.import_module("__graft_entry__")
        opts = {"setup": list(worker_setup),
                "install": {"fuse_qk_epilogue": fuse_qk_epilogue, "fuse_sampler": fuse_sampler,
                            "device_metadata": device_metadata, "fuse_row_parallel": fuse_row_parallel,
                            "row_parallel_allreduce": row_parallel_allreduce}}
        engine_mod.ModelRunner = functools.partial(entry.nanovllm_worker, options=opts)
    else:
        engine_mod.ModelRunner = runner_mod.ModelRunner
    return attn_mod, qwen3


def uninstall():
    """Point Attention back at this package's own context mirror."""
    from . import context as _ctx
    _attention.set_context_source(_ctx.get_context)
