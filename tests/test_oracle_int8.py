"""The oracle's w8a8 quantisation rules on hand-checked values (CPU)."""
import numpy as np

from oracle import rwkv


def test_quantize_rows_known_values():
    x = np.array([[1.0, -2.0, 0.5, 0.0], [0, 0, 0, 0], [3.0, 1.5, -0.75, 0.01]], np.float32)
    q, s = rwkv.quantize_rows(x)
    # row 0: amax 2 -> 127/2 = 63.5; 1*63.5 = 63.5 -> 64 (half to even), 0.5*63.5 = 31.75 -> 32
    assert q[0].tolist() == [64, -127, 32, 0]
    assert s[0] == np.float32(2.0) / np.float32(127)
    assert q[1].tolist() == [0, 0, 0, 0] and s[1] == 0
    # row 2: amax 3 -> 42.333...; 1.5 -> 63.5 rounded in fp32 arithmetic
    inv = np.float32(127) / np.float32(3.0)
    assert q[2].tolist() == [127, int(np.rint(np.float32(1.5) * inv)),
                             int(np.rint(np.float32(-0.75) * inv)),
                             int(np.rint(np.float32(np.float16(0.01)) * inv))]


def test_quantize_weight_per_output_channel():
    W = np.array([[0.5, -0.01], [-1.0, 0.02], [0.25, 0.0]], np.float32)  # [in=3, out=2]
    q, s = rwkv.quantize_weight(W)
    assert q.shape == (2, 3) and s.dtype == np.float16
    assert s[0] == np.float16(np.float32(1.0) / np.float32(127))
    assert q[0, 1] == -127 and abs(int(q[0, 0]) - 64) <= 1
    assert q[1, 1] == 127


def test_i8_forward_close_to_fp32():
    from krunch_b200.synth import random_weights
    w = random_weights(2, 128, 512, 300, seed=1)
    tok = np.random.default_rng(0).integers(0, 300, (1, 6))
    a, _ = rwkv.forward(w, tok)
    b, _ = rwkv.forward(w, tok, wdtype="i8")
    assert np.abs(a - b).max() < 0.05
