"""Generate tests/golden/decode_meta.npz from the reference's own decode-step builders.

Runs nano-vLLM's ModelRunner.prepare_decode, prepare_block_tables and prepare_sample
(nanovllm/engine/model_runner.py:123-127, :167-193) on CPU over real reference
Sequence objects (nanovllm/engine/sequence.py) with seeded lengths, last tokens,
temperatures and block tables.  The builders' pinned-memory host tensors and
.cuda() copies are made no-ops for the run (there is no GPU here); nothing else is
changed.  Records every sequence's inputs and the tensors the builders returned or
put in the context.  Needs the reference checkout (its directory as argv[1] or in
NANOVLLM_REF); run once in the development container, output committed.

Usage:  python tests/golden/gen_decode_meta_golden.py [REF_DIR]
"""
import os
import sys

os.environ.setdefault("TORCH_COMPILE_DISABLE", "1")
import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NANOVLLM_REF", "")
if not os.path.isdir(os.path.join(REF, "nanovllm")):
    sys.exit(__doc__)
sys.path.insert(0, REF)
from nanovllm.engine import model_runner  # noqa: E402
from nanovllm.engine.sequence import Sequence  # noqa: E402
from nanovllm.sampling_params import SamplingParams  # noqa: E402
from nanovllm.utils.context import get_context  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_meta.npz")


def host_only():
    """torch.tensor without pinned memory and Tensor.cuda as identity, for the builders."""
    real_tensor = torch.tensor

    def tensor(*args, **kwargs):
        kwargs.pop("pin_memory", None)
        return real_tensor(*args, **kwargs)

    model_runner.torch.tensor = tensor
    torch.Tensor.cuda = lambda self, *a, **k: self


def make_seqs(rng, B, max_len, pool):
    ids = rng.permutation(pool)  # distinct block ids across the batch
    seqs, used = [], 0
    for _ in range(B):
        n = int(rng.integers(1, max_len + 1))
        sp = SamplingParams(temperature=float(rng.uniform(0.1, 2.0)))
        s = Sequence([int(t) for t in rng.integers(0, 151936, size=1)], sp)
        # a decode-time sequence: n tokens, the last one given; blocks for all n
        s.num_tokens = n
        s.last_token = int(rng.integers(0, 151936))
        nb = (n + Sequence.block_size - 1) // Sequence.block_size
        s.block_table = [int(b) for b in ids[used:used + nb]]
        used += nb
        seqs.append(s)
    return seqs


def run_case(name, B, max_len, pool, seed, store):
    rng = np.random.default_rng(seed)
    seqs = make_seqs(rng, B, max_len, pool)
    runner = object.__new__(model_runner.ModelRunner)
    runner.block_size = Sequence.block_size
    input_ids, positions = model_runner.ModelRunner.prepare_decode(runner, seqs)
    temps = model_runner.ModelRunner.prepare_sample(runner, seqs)
    ctx = get_context()
    store[name + ".lengths"] = np.array([len(s) for s in seqs], np.int64)
    store[name + ".last_tokens"] = np.array([s.last_token for s in seqs], np.int64)
    store[name + ".temperatures_in"] = np.array([s.temperature for s in seqs], np.float64)
    store[name + ".table_offsets"] = np.cumsum([0] + [len(s.block_table) for s in seqs]).astype(np.int64)
    store[name + ".tables_flat"] = np.array([b for s in seqs for b in s.block_table], np.int64)
    store[name + ".input_ids"] = input_ids.numpy()
    store[name + ".positions"] = positions.numpy()
    store[name + ".slot_mapping"] = ctx.slot_mapping.numpy()
    store[name + ".context_lens"] = ctx.context_lens.numpy()
    store[name + ".block_tables"] = ctx.block_tables.numpy()
    store[name + ".temperatures"] = temps.numpy()


def main():
    host_only()
    store = {}
    run_case("b1", 1, 300, 64, 1, store)
    run_case("b17_short", 17, 256, 512, 2, store)
    run_case("b64_mixed", 64, 4096, 2048, 3, store)
    run_case("b256_long", 256, 12000, 16384, 4, store)
    np.savez_compressed(OUT, **store)
    print(OUT, len(store))


if __name__ == "__main__":
    main()
