"""CPU: the FSQ host helpers of the library (acb_fsq_decode_index / acb_fsq_encode_index) against
the oracle's restatement of fsq_decode_index (src/fsq-detok.h:18-29) and fsq_encode_index
(src/fsq-tok.h:42-60): every one of the 64000 codes decodes bit-identically, codes survive a
decode -> atanh -> encode round trip, and random pre-activations encode to the same index."""
import numpy as np

import acb
import oracle as O


def test_fsq_decode_every_code():
    for code in range(0, 64000, 1):
        a = acb.fsq_decode_index(code)
        b = O.fsq_decode_index(code)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), code


def test_fsq_levels_and_range():
    lo = O.fsq_decode_index(0)
    hi = O.fsq_decode_index(63999)
    assert np.all(lo == -1.0) and np.all(hi == 1.0)


def test_fsq_encode_round_trip_and_random():
    rng = np.random.default_rng(5)
    for code in rng.integers(0, 64000, 2000):
        x = O.fsq_decode_index(int(code))
        # values strictly inside (-1, 1) pulled back through tanh land on their own level
        raw = np.arctanh(np.clip(x, -0.999, 0.999)).astype(np.float32)
        assert O.fsq_encode_index(raw) == code
        assert acb.fsq_encode_index(raw) == code
    for _ in range(2000):
        raw = (rng.standard_normal(6) * 1.5).astype(np.float32)
        assert acb.fsq_encode_index(raw) == O.fsq_encode_index(raw)
