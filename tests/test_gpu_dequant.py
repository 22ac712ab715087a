"""Device weight decoding against the reference's golden vectors, bit for bit.

quant_k_test.go:14-48 pins the Go decoder (decodeKBlock, quant_k.go:31-86) to
gguf's float32 values for 4 x 2048 weights of each format, including reads
that start and end inside a block. The same fixtures are checked here through
every decoder the CUDA kernels use, via tcu_read_values:

  element  the per-element decoder of the matrix-vector kernels (all formats)
  group8   the 8-value decoder of the batched products (Q6_K, Q5_K)
  tc       the tcgen05 GEMM operand: binary16 pieces summed back (Q8_0, Q6_K, Q5_K)

Q8_0 has no reference fixture; tests/golden/kquant/q8_0*.bin holds gguf's
quantiser output and its own dequantisation (make_golden.py).
"""
import numpy as np
import pytest

from tinyoai_b200 import BackendError, _lib, read_values

pytestmark = pytest.mark.gpu

FIXTURES = {"q5_k": "Q5_K", "q6_k": "Q6_K", "q5_1": "Q5_1", "q8_0": "Q8_0"}
DECODERS = {"Q5_K": ("element", "group8", "tc"), "Q6_K": ("element", "group8", "tc"), "Q5_1": ("element",),
            "Q8_0": ("element", "tc")}
PARTIAL = [(0, 1), (255, 3), (257, 511), (1000, 777), (8191, 1)]


def load(golden, name):
    raw = (golden / "kquant" / f"{name}.bin").read_bytes()
    want = np.frombuffer((golden / "kquant" / f"{name}-f32.bin").read_bytes(), dtype="<u4")
    return raw, want


@pytest.mark.parametrize("name", list(FIXTURES))
def test_decoders_bitwise(golden, name):
    dtype = FIXTURES[name]
    raw, want = load(golden, name)
    for dec in DECODERS[dtype]:
        got = read_values(dtype, raw, 4, 2048, decoder=dec)
        bad = np.nonzero(got.view(np.uint32) != want)[0]
        assert bad.size == 0, f"{dec}: {bad.size} values differ, first at {bad[0]}"
        for start, n in PARTIAL:
            part = read_values(dtype, raw, 4, 2048, offset=start, n=n, decoder=dec)
            assert np.array_equal(part.view(np.uint32), want[start:start + n]), (dec, start, n)


def test_dense_formats_bitwise():
    """BF16 (bits << 16) and F16 (IEEE binary16) element decode, every bit
    pattern of binary16 and a seeded spread of bfloat16."""
    h = np.arange(65536, dtype=np.uint16)
    got = read_values("F16", h.tobytes(), 256, 256)
    want = h.view(np.float16).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    b = np.random.default_rng(5).integers(0, 65536, 64 * 128, dtype=np.uint32).astype(np.uint16)
    got = read_values("BF16", b.tobytes(), 64, 128)
    assert np.array_equal(got.view(np.uint32), b.astype(np.uint32) << 16)


def test_read_values_rejects_bad_requests(golden):
    raw, _ = load(golden, "q6_k")
    for kwargs in (dict(offset=8190, n=3), dict(offset=-1, n=1)):
        with pytest.raises(BackendError) as e:
            read_values("Q6_K", raw, 4, 2048, **kwargs)
        assert e.value.code == _lib.TCU_EINVAL
    with pytest.raises(BackendError) as e:
        read_values("Q6_K", raw[:-1], 4, 2048)
    assert e.value.code == _lib.TCU_EINVAL
    raw1, _ = load(golden, "q5_1")
    with pytest.raises(BackendError) as e:
        read_values("Q5_1", raw1, 4, 2048, decoder="tc")
    assert e.value.code == _lib.TCU_EUNSUP
