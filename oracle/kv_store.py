"""KV-cache scatter oracle (test infrastructure only).

Restates `store_kvcache` / `store_kvcache_kernel` of
nanovllm/layers/attention.py:10-40: for every token row t with
slot_mapping[t] != -1, the Hkv*D contiguous elements of key[t] and value[t]
are copied to row slot_mapping[t] of the flat caches
k_cache.view(-1, Hkv*D) / v_cache.view(-1, Hkv*D).  The copy is bitwise.
"""
import numpy as np


def check_store_args(key, value, k_cache, v_cache, slot_mapping):
    """The launcher asserts of nanovllm/layers/attention.py:35-39, on shapes.

    numpy arrays carry byte strides; the reference checks element strides of
    torch tensors: stride(-1) == 1, stride(1) == head_dim, cache row stride
    == Hkv*head_dim and numel(slot_mapping) == N.
    """
    n, hkv, d = key.shape
    item = key.itemsize
    assert key.strides[-1] == item and value.strides[-1] == item
    assert key.strides[1] == d * item and value.strides[1] == d * item
    assert k_cache.strides[1] == hkv * d * item and v_cache.strides[1] == hkv * d * item
    assert slot_mapping.size == n


def store_kvcache_ref(key, value, k_cache, v_cache, slot_mapping):
    """Vectorised scatter, in place on k_cache / v_cache.

    key, value: [N, Hkv, D] (any row stride); caches [NB, block_size, Hkv, D]
    contiguous; slot_mapping int32 [N].  Slots outside [0, NB*block_size) are
    skipped like -1 (the reference would write out of bounds; the CUDA kernel
    skips them, so the oracle does too).  Non-negative slots are expected to
    be unique (nanovllm never issues duplicates; the Triton kernel leaves the
    winner of a duplicate undefined).
    """
    check_store_args(key, value, k_cache, v_cache, slot_mapping)
    n, hkv, d = key.shape
    row = hkv * d
    kf = k_cache.reshape(-1, row)
    vf = v_cache.reshape(-1, row)
    slots = np.asarray(slot_mapping, dtype=np.int64)
    ok = (slots >= 0) & (slots < kf.shape[0])
    kf[slots[ok]] = key.reshape(n, row)[ok]
    vf[slots[ok]] = value.reshape(n, row)[ok]


def store_kvcache_loop_ref(key, value, k_cache, v_cache, slot_mapping, block_size):
    """Per-token loop form of the same contract (small cases only).

    Follows the slot -> (block, offset) decomposition of the study guide's
    store contract (master_nano-vllm-v2.md:2807-2852): block = slot //
    block_size, offset = slot % block_size, cache[block, offset] = row.
    """
    nb = k_cache.shape[0]
    for t in range(key.shape[0]):
        slot = int(slot_mapping[t])
        if slot < 0 or slot >= nb * block_size:
            continue
        blk, off = divmod(slot, block_size)
        k_cache[blk, off] = key[t]
        v_cache[blk, off] = value[t]
