"""Sparse-attention output projection with the post-attention hc expand
(NativePrefillDSAOutputPlan, native_execution/native_prefill_dsa_output_plan.h).
The layout step is bit-exact; the projection is block_fp8_linear (the layer
bar: max(2e-2, 1 BF16 ulp), cosine >= 0.9999 against the oracle); execute_hc
equals hc_expand of execute bit for bit."""

import numpy as np
import pytest
import torch

from gpu_util import assert_layer_close, bits, certify_linear, from_bits


def test_oracle_layout_known_answer(oracle):
    hm = np.arange(2 * 3 * 8, dtype=np.uint16).reshape(2, 3, 8)
    rows = oracle.head_major_to_rows(hm)
    assert rows.shape == (3, 16)
    np.testing.assert_array_equal(rows[1, :8], hm[0, 1])
    np.testing.assert_array_equal(rows[1, 8:], hm[1, 1])
    np.testing.assert_array_equal(rows, hm.transpose(1, 0, 2).reshape(3, 16))


def _weights(N, K, seed, dev):
    from glm53_flash_mlx_b200 import synthetic as S

    return S.random_block_fp8(N, K, seed=seed, device=dev)


@pytest.mark.gpu
@pytest.mark.parametrize("heads,rows,dim", [(64, 256, 256), (3, 5, 24), (1, 1, 8)])
def test_head_major_to_rows_bit_exact(oracle, heads, rows, dim):
    import glm53_flash_mlx_b200 as G

    rng = np.random.default_rng(heads * rows + dim)
    hm = rng.integers(0, 1 << 16, size=(heads, rows, dim), dtype=np.uint16)
    out = G.head_major_to_rows(from_bits(hm, "cuda"))
    np.testing.assert_array_equal(bits(out), oracle.head_major_to_rows(hm))


@pytest.mark.gpu
@pytest.mark.parametrize("heads,rows,dim,hidden,check_rows", [(4, 19, 128, 256, None),
                                                               (64, 256, 256, 4096, [0, 77, 255])])
def test_dsa_output_projection_and_hc(oracle, heads, rows, dim, hidden, check_rows):
    import glm53_flash_mlx_b200 as G

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(rows + hidden)
    hm = oracle.bf16_from_f32(rng.standard_normal((heads, rows, dim)).astype(np.float32))
    w, s = _weights(hidden, heads * dim, seed=rows, dev=dev)
    plan = G.DSAOutputProjection()
    hm_d = from_bits(hm, dev)
    projected = plan.execute(hm_d, w, s)
    row_major = G.head_major_to_rows(hm_d)
    assert torch.equal(projected, G.block_fp8_linear(row_major, w, s))
    sel = list(range(rows)) if check_rows is None else check_rows
    rows_in = oracle.head_major_to_rows(hm)[sel]
    ref = oracle.block_fp8_linear(rows_in, w.cpu().numpy(), s.cpu().numpy())
    cert = certify_linear(rows_in, w.cpu().numpy(), s.cpu().numpy(), bits(projected)[sel])
    assert_layer_close(bits(projected)[sel], ref, certificate=cert)
    residual = oracle.bf16_from_f32(rng.standard_normal((rows, 4, hidden)).astype(np.float32))
    post = (rng.random((rows, 4)) * 2).astype(np.float32)
    comb = rng.random((rows, 4, 4)).astype(np.float32)
    args = (from_bits(residual, dev), torch.from_numpy(post).to(dev), torch.from_numpy(comb).to(dev))
    out = plan.execute_hc(hm_d, w, s, *args)
    assert torch.equal(out, G.hc_expand(projected, *args))
    np.testing.assert_array_equal(bits(out), oracle.hc_expand(bits(projected), residual, post, comb))
    assert plan.execution_count == 2


@pytest.mark.gpu
def test_dsa_output_rejects_mismatched_weight():
    import glm53_flash_mlx_b200 as G

    dev = torch.device("cuda:0")
    w, s = _weights(256, 512, seed=1, dev=dev)
    with pytest.raises(ValueError, match="does not take"):
        G.DSAOutputProjection().execute(torch.zeros((2, 8, 128), dtype=torch.bfloat16, device=dev), w, s)
    with pytest.raises(ValueError, match="multiple of 8"):
        G.head_major_to_rows(torch.zeros((2, 3, 12), dtype=torch.bfloat16, device=dev))
