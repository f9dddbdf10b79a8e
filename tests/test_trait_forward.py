"""The reference's decode forward (BitNetModel::forward_into,
crates/bitnet-model/src/lib.rs:931-1163) driven from C through the
host-slice entry points alone, one trait call per reference call
(tests/trait_forward.c): what the Rust CudaBackend shim does when the
reference model calls it op by op.  The harness builds against
include/bitnet_cuda.h and libbitnet_cuda.so on the CPU; on a GPU its logits
must be bit-identical to the oracle's forward at every position."""
import shutil
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import ModelConfig, synth

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "bitnetrs_b200"
CFG = ModelConfig(512, 256, 2, 8, 2, 384, 64, 500000.0, 1e-5)
TOKENS = [3, 141, 59, 265, 358, 97, 11, 500]


def build_harness(out_dir: Path) -> Path:
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    if not (LIBDIR / "libbitnet_cuda.so").exists():
        pytest.fail("libbitnet_cuda.so is missing: build it first (python -m bitnetrs_b200.build)")
    exe = out_dir / "trait_forward"
    subprocess.run([gcc, "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror", "-ffp-contract=off",
                    "-I", str(ROOT / "include"), str(ROOT / "tests" / "trait_forward.c"), "-o", str(exe),
                    "-L", str(LIBDIR), "-lbitnet_cuda", f"-Wl,-rpath,{LIBDIR}", "-Wl,--allow-shlib-undefined"],
                   check=True, capture_output=True, text=True)
    return exe


def write_model(path: Path, w, tokens):
    c = w.config
    with open(path, "wb") as f:
        f.write(b"BNTF" + struct.pack("<I", 1))
        f.write(struct.pack("<7I", c.vocab_size, c.hidden_size, c.num_hidden_layers, c.num_attention_heads,
                            c.num_key_value_heads, c.intermediate_size, c.max_position_embeddings))
        f.write(struct.pack("<2f", c.rope_theta, c.rms_norm_eps))
        for L in w.layers:
            for proj, scale in ((L.q_proj, L.q_scale), (L.k_proj, L.k_scale), (L.v_proj, L.v_scale),
                                (L.o_proj, L.o_scale), (L.gate_proj, L.gate_scale), (L.up_proj, L.up_scale),
                                (L.down_proj, L.down_scale)):
                b = np.ascontiguousarray(proj, dtype=np.uint8).tobytes()
                f.write(struct.pack("<Q", len(b)) + b + struct.pack("<f", scale))
            for norm in (L.attention_norm, L.attn_sub_norm, L.ffn_norm, L.ffn_sub_norm):
                f.write(np.ascontiguousarray(norm, dtype=np.float32).tobytes())
        f.write(np.ascontiguousarray(w.embed_tokens, dtype=np.uint16).tobytes())
        f.write(np.ascontiguousarray(w.lm_head_i8, dtype=np.int8).tobytes())
        f.write(np.ascontiguousarray(w.lm_head_scales, dtype=np.float32).tobytes())
        f.write(np.ascontiguousarray(w.final_norm, dtype=np.float32).tobytes())
        f.write(struct.pack("<I", len(tokens)) + np.asarray(tokens, dtype=np.uint32).tobytes())


def test_trait_harness_builds(tmp_path):
    """The C harness compiles against the header (C99, warnings as errors)
    and links against the library: the whole per-op path a C or Rust caller
    needs is declared and exported."""
    exe = build_harness(tmp_path)
    assert exe.exists()


@pytest.mark.gpu
def test_trait_forward_matches_oracle(tmp_path):
    exe = build_harness(tmp_path)
    w = synth.random_model(CFG, seed=5)
    model = tmp_path / "model.bin"
    out = tmp_path / "logits.bin"
    write_model(model, w, TOKENS)
    res = subprocess.run([str(exe), str(model), str(out)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    got = np.fromfile(out, dtype=np.float32).reshape(len(TOKENS), CFG.vocab_size)
    om = O.OracleModel(w)
    okv = om.kv(len(TOKENS))
    for pos, tok in enumerate(TOKENS):
        ref = om.forward(okv, [tok], pos)
        np.testing.assert_array_equal(got[pos], ref, err_msg=f"position {pos}")
