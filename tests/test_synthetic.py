"""The benchmark's synthetic checkpoint and audio (lbrr.synthetic) are the very
tensors the parity tests feed the oracle, so a bench run measures the inputs
parity was shown on; and the checkpoint passes the loader's full validation."""
import numpy as np

import lbrr
from lbrr import synthetic
from oracle import bsroformer_ref as R


def test_checkpoint_matches_oracle_generator():
    a = synthetic.checkpoint(seed=5, gamma_noise=0.1)
    b = R.make_weights(seed=5, gamma_noise=0.1)
    assert list(a) == list(b)
    assert [tuple(v.shape) for v in a.values()] == [s for _, s in R.weight_keys()]
    for k in a:
        assert np.array_equal(a[k].numpy(), b[k].numpy()), k
    lbrr.check_weights(a)


def test_audio_matches_oracle_generator():
    for n, seed in ((1, 0), (4096, 7), (100003, 42)):
        x = synthetic.audio(n, seed)
        assert x.shape == (2, n) and x.dtype == np.float32
        assert np.array_equal(x, R.synth_audio(n, seed))
