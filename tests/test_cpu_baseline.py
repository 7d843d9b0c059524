"""The timed CPU baseline (oracle/msb_cpu_fast.c: ggml's q8_0 mul_mat_id
restated with vectorized int8 dots, threaded) against the scalar oracle in
the same q8 form. The f32 lane sums run in another order, and a re-quantized
SwiGLU output can round a code differently, so the FFN agrees to 1e-3 of the
output's max, not bit for bit."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import experts, topk_ids

ISAS = [i for i in (0, 1, 2) if i <= {"scalar": 0, "avx2": 1, "avx512-vnni": 2}[O.fast_isa()]]


@pytest.mark.parametrize("isa", ISAS)
@pytest.mark.parametrize("wtype,K,n_ff,n_expert,n_tok,top_k,fused,act", [
    ("mxfp4", 2880, 2880, 6, 5, 4, True, None),        # gpt-oss widths, fused gate_up
    ("mxfp4", 512, 256, 8, 40, 4, False, (1.702, 7.0)),  # many pairs per slot, gpt-oss act
    ("iq4_nl", 2048, 512, 10, 8, 8, False, None),      # 256-expert model widths
    ("iq4_nl", 96, 64, 4, 3, 2, True, None),           # odd block count
])
def test_fast_ffn_matches_scalar_q8(isa, wtype, K, n_ff, n_expert, n_tok, top_k, fused, act):
    try:
        O.fast_isa(isa)
        rng = np.random.default_rng(K + n_tok)
        if fused:
            gate = up = experts(wtype, n_expert, K, 2 * n_ff, seed=1)
            up_row0 = n_ff
        else:
            gate = experts(wtype, n_expert, K, n_ff, seed=1)
            up = experts(wtype, n_expert, K, n_ff, seed=2)
            up_row0 = 0
        down = experts(wtype, n_expert, n_ff, K, seed=3)
        x = rng.normal(0, 2, size=(n_tok, K)).astype(np.float32)
        ids, w = topk_ids(rng, n_tok, n_expert, top_k)
        want, _ = O.moe_ffn(wtype, gate, up, down, K, n_ff, x, ids, w, mode="q8",
                            up_row0=up_row0, act=act)
        got = O.moe_ffn_fast(wtype, gate, up, down, K, n_ff, x, ids, w, up_row0=up_row0,
                             act=act, nthreads=3)
        assert O.max_abs_normalized(got, want) < 1e-3
    finally:
        O.fast_isa(-1)
