"""Weight-only FP8 (E4M3) quantization on the CPU: the oracle's encoder agrees
with torch's float8_e4m3fn rounding, and the library's quantizer (which the
model runs at load time) agrees with the oracle's bit for bit."""
import numpy as np
import pytest

from helpers import load_oracle, load_pkg

O = load_oracle()
pkg = load_pkg()


def test_oracle_e4m3_matches_torch_rounding():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 100, 20000), rng.normal(0, 0.01, 20000), rng.uniform(-448, 448, 20000),
                        np.ldexp(rng.integers(-1024, 1024, 5000), -13)]).astype(np.float32)
    L = O.lib()
    ours = np.array([L.oracle_e4m3_encode(float(v)) for v in x], dtype=np.uint8)
    ref = torch.from_numpy(x).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)
    codes = [c for c in range(256) if (c & 0x7F) != 0x7F]
    dec = np.array([L.oracle_e4m3_decode(c) for c in codes], dtype=np.float32)
    tdec = torch.tensor(codes, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(dec, tdec)


@pytest.mark.parametrize("K,N", [(768, 2304), (1600, 37), (64, 1)])
def test_library_quantizer_matches_oracle(K, N):
    rng = np.random.default_rng(K + N)
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    w[3, 0] = 0.9      # an outlier sets its column's scale
    if N > 2:
        w[:, 2] = 0.0  # an all-zero column
    q1, s1 = pkg.fp8_quantize(w)
    q2, s2 = O.fp8_quantize(w)
    assert np.array_equal(q1, q2)
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    assert np.all(s1 > 0)
