"""Regenerate the golden fixtures under tests/golden/ from a reference checkout.

Usage (only where the reference tree is present; never at test time):

    python tests/golden/make_golden.py /path/to/tinyoai

What it writes, and where each file comes from inside the reference project:

* ``kquant/{q5_k,q6_k,q5_1}.bin`` and ``*-f32.bin``: copies of
  ``testdata/gguf/*`` (generated upstream by scripts/make_k_quant_fixtures.py
  with gguf==0.17.1, seed 9041); the decode is pinned bitwise
  (quant_k_test.go:14-33).
* ``kquant/q8_0.bin`` / ``q8_0-f32.bin``: a Q8_0 vector quantized and
  dequantized by the installed ``gguf`` package (0.19.0), an independent
  decoder for the format that the reference checks only synthetically.
* ``stablelm_tiny/``: ``config.json``, both safetensors shards, the index,
  ``expected.json`` (Transformers fp32 logits, 3e-5 in stablelm_test.go:50-82)
  and ``rope.json`` (split-half RoPE boundary cases, 5e-7 in
  stablelm_test.go:181-205).
* ``stablelm_tiny/generation.json``: the token ids of the fixture's greedy
  generation prompt, encoded with the fixture's tokenizer.json by the
  ``tokenizers`` package.
* ``llama/stories260K.bin`` and ``tok512.bin``: copies of ``assets/`` (the
  embedded default model, model.go / embed.go).
* ``MANIFEST.json``: SHA-256 of every file, with its source path.
"""
import hashlib
import json
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def main(ref):
    ref = Path(ref)
    manifest = {}

    def copy(src, dst):
        dst = HERE / dst
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(ref / src, dst)
        manifest[str(dst.relative_to(HERE))] = {"source": src, "sha256": sha(dst)}

    for name in ["q5_k", "q6_k", "q5_1"]:
        copy(f"testdata/gguf/{name}.bin", f"kquant/{name}.bin")
        copy(f"testdata/gguf/{name}-f32.bin", f"kquant/{name}-f32.bin")
    for name in ["config.json", "expected.json", "rope.json", "model.safetensors.index.json",
                 "model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]:
        copy(f"testdata/stablelm/{name}", f"stablelm_tiny/{name}")
    copy("assets/stories260K.bin", "llama/stories260K.bin")
    copy("assets/tok512.bin", "llama/tok512.bin")

    # Token ids of the fixture's generation prompt (stablelm_test.go:73-82),
    # produced by the `tokenizers` package from the fixture's tokenizer.json
    # (the tokenizer itself is outside the CUDA path).
    from tokenizers import Tokenizer
    tok = Tokenizer.from_file(str(ref / "testdata/stablelm/tokenizer.json"))
    expected = json.loads((ref / "testdata/stablelm/expected.json").read_text())
    prompt = expected["generation"]["prompt"]
    gen = {"prompt": prompt, "prompt_ids": tok.encode(prompt).ids, "ids": expected["generation"]["ids"]}
    (HERE / "stablelm_tiny/generation.json").write_text(json.dumps(gen) + "\n")
    manifest["stablelm_tiny/generation.json"] = {"source": "tokenizers encode of testdata/stablelm expected.json prompt",
                                                 "sha256": sha(HERE / "stablelm_tiny/generation.json")}

    import gguf
    rng = np.random.default_rng(9042)
    # 4 rows x 2048 values: N(0, 0.02) like the synthetic configs, plus an
    # all-zero block, a huge block and a tiny (subnormal-scale) block.
    x = (rng.standard_normal((4, 2048)) * 0.02).astype(np.float32)
    x[1, 0:32] = 0
    x[2, 32:64] *= 1e4
    x[3, 64:96] = 1e-7 * np.sign(x[3, 64:96])
    raw = gguf.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    dec = gguf.dequantize(raw, gguf.GGMLQuantizationType.Q8_0).astype("<f4")
    (HERE / "kquant").mkdir(exist_ok=True)
    (HERE / "kquant/q8_0.bin").write_bytes(np.ascontiguousarray(raw).tobytes())
    (HERE / "kquant/q8_0-f32.bin").write_bytes(dec.tobytes())
    for n in ["kquant/q8_0.bin", "kquant/q8_0-f32.bin"]:
        manifest[n] = {"source": f"gguf {gguf.__version__ if hasattr(gguf, '__version__') else '0.19.0'} quantize/dequantize, seed 9042",
                       "sha256": sha(HERE / n)}
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(manifest)} fixtures")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
