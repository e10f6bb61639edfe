"""Generate the golden fixtures in this folder from the reference's own code.

Run in a container where the reference checkout is present (it is not needed at
test time):

    python tests/golden/make_golden.py /path/to/hotschmoe-xe2x2

It imports kernels/nvfp4/gptq_s4_dump.py (numpy only; its main() is guarded) and
records, for seeded random packed words, the outputs of the reference's
checkpoint unpackers unpack_i32_nibbles_first (qweight, :69-73) and
unpack_i32_nibbles_last (qzeros, :61-66), plus the reference's s4 view u - 8
(:114).  tests/test_oracle_golden.py replays them against the C oracle.

It also writes a tiny act_order GPTQ checkpoint with this repository's
safetensors writer (gptq_tiny.safetensors, seeded values) and records what the
reference's own reader load_meta / read_tensor (:32-58) returns for every
tensor in it (gptq_tiny_ref.npz); tests/test_checkpoint.py reads the same file
with xe2x2_b200.checkpoint and compares.  Finally it runs the reference's own
main() on that checkpoint, which writes its tile dumps gptq_tiny_s4.bin and
gptq_tiny_s4_sc.bin (:153-181).
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np


def main(ref_root: str) -> None:
    path = os.path.join(ref_root, "kernels", "nvfp4", "gptq_s4_dump.py")
    spec = importlib.util.spec_from_file_location("gptq_s4_dump", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    rng = np.random.default_rng(20261201)
    out = {}
    for name, (rows, cols) in {"a": (16, 40), "b": (64, 24)}.items():
        qw = rng.integers(-2**31, 2**31, size=(rows, cols), dtype=np.int64).astype(np.int32)
        qz = rng.integers(-2**31, 2**31, size=(rows // 8 + 1, cols // 8 + 1), dtype=np.int64).astype(np.int32)
        out[f"{name}_qweight"] = qw
        out[f"{name}_unpack_first"] = mod.unpack_i32_nibbles_first(qw).astype(np.int16)
        out[f"{name}_s4"] = (mod.unpack_i32_nibbles_first(qw).astype(np.int16) - 8).astype(np.int16)
        out[f"{name}_qzeros"] = qz
        out[f"{name}_unpack_last"] = mod.unpack_i32_nibbles_last(qz).astype(np.int16)
    here = os.path.dirname(os.path.abspath(__file__))
    np.savez_compressed(os.path.join(here, "gptq_unpack.npz"), **out)
    print("wrote", os.path.join(here, "gptq_unpack.npz"), sorted(out))

    path = os.path.join(here, "gptq_tiny.safetensors")
    write_tiny_checkpoint(path)
    meta, data0 = mod.load_meta(path)
    ref = {name: mod.read_tensor(path, data0, info) for name, info in meta.items()}
    np.savez_compressed(os.path.join(here, "gptq_tiny_ref.npz"), **ref)
    print("wrote", path, "and gptq_tiny_ref.npz", sorted(ref))

    # the reference's own tile dumps of that checkpoint (its main(): plain and scaled forms)
    env = {"GPTQ_ST": path, "GPTQ_DUMP": os.path.join(here, "gptq_tiny_s4.bin"),
           "GPTQ_DUMP_SC": os.path.join(here, "gptq_tiny_s4_sc.bin"), "TILE_K": "128", "TILE_N": "64"}
    old_env = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        spec = importlib.util.spec_from_file_location("gptq_s4_dump_main", os.path.join(ref_root, "kernels", "nvfp4",
                                                                                       "gptq_s4_dump.py"))
        dump_mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(dump_mod)  # reads the env at import
        rc = dump_mod.main()
    finally:
        for k, v in old_env.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    print("reference dump main() ->", rc)


def tiny_checkpoint_tensors() -> dict:
    """One act_order GPTQ layer, K=128, N=64, group 32, asymmetric zeros (seeded)."""
    rng = np.random.default_rng(20261202)
    K, N, gs = 128, 64, 32
    qw = rng.integers(-2**31, 2**31, size=(K // 8, N), dtype=np.int64).astype(np.int32)
    qz = rng.integers(-2**31, 2**31, size=(K // gs, N // 8), dtype=np.int64).astype(np.int32)
    sc = (np.abs(rng.normal(0, 0.02, size=(K // gs, N))) + 1e-3).astype(np.float16)
    g_idx = rng.permutation(np.arange(K, dtype=np.int32) // gs).astype(np.int32)
    p = "model.layers.0.mlp.down_proj"
    return {p + ".qweight": qw, p + ".qzeros": qz, p + ".scales": sc, p + ".g_idx": g_idx}


def write_tiny_checkpoint(path: str) -> None:
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    from xe2x2_b200.checkpoint import save_safetensors

    save_safetensors(path, tiny_checkpoint_tensors(), metadata={"format": "pt"})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout root>")
    main(sys.argv[1])
