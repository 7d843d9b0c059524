"""Device quantizers are bit-identical to the oracle's (MXFP4 follows the
gguf quantizer; IQ4_NL this library's scale search)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wtype", ["mxfp4", "iq4_nl"])
def test_device_quantizer_matches_oracle(wtype):
    from moestream_b200 import ops
    rng = np.random.default_rng(0)
    x = rng.normal(0, 0.02, size=(96, 2880)).astype(np.float32)
    x[0, :32] = 0.0            # all-zero block
    x[1, :32] = 1.0            # constant block
    x[2, :32] *= 1e4           # large scale
    x[3, 5] = -3.0             # single outlier
    got = ops.quantize_rows(wtype, torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    want = O.quantize(wtype, x)
    assert np.array_equal(got.cpu().numpy(), want)
