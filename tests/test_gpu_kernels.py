"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Quantiser: bit-exact (codes and scale bits). GEMMs: relative Frobenius error <= 5e-3
against the fp64-accumulated oracle on the oracle-decoded weights,
plus an elementwise bound of a few bf16 ulps of the output scale.
"""

from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200 import quant_kernels as qk
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3
TORCH_OF = {O.F16: torch.float16, O.BF16: torch.bfloat16, O.F32: torch.float32}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.detach().cpu().numpy()


def _status_ok(device):
    assert qk.check_device_status(device) & _lib.STATUS_TIMEOUT_MASK == 0


# ------------------------------------------------------------------------------- quantiser
@pytest.mark.parametrize("name", ["q_70x37_f32", "q_64x32_zero_row", "q_96x40_bf16", "q_48x24_f16", "q_ties"])
def test_quantiser_bit_exact_on_golden_weights(cuda_device, golden_arrays, name):
    w = torch.from_numpy(golden_arrays[f"{name}.w"]).to(cuda_device)
    q, s = qk.quantize_weight(w)
    np.testing.assert_array_equal(q.cpu().numpy(), golden_arrays[f"{name}.q"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), golden_arrays[f"{name}.s"].view(np.uint32))


@pytest.mark.parametrize("shape", [(3072, 3072), (12288, 3072), (3072, 12288), (18432, 3072), (16384, 3072),
                                   (3072, 8192)])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_quantiser_bit_exact_at_baseline_shapes(cuda_device, golden_meta, shape, dtype):
    out_f, in_f = shape
    gen = torch.Generator().manual_seed(0)
    w = (torch.randn(out_f, in_f, generator=gen) * 0.02).to(getattr(torch, dtype))
    expected = golden_meta["quant_hash"][f"{out_f}x{in_f}:{dtype}"]
    q, s = qk.quantize_weight(w.to(cuda_device))
    assert sha(q.cpu().numpy()) == expected["codes_sha256"]
    assert sha(s.cpu().numpy()) == expected["scale_sha256"]


@pytest.mark.parametrize("src_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_quantiser_matches_oracle_on_random_ragged_shapes(cuda_device, src_dtype):
    gen = torch.Generator().manual_seed(3)
    for n, k in [(1, 1), (5, 33), (129, 257), (300, 1000)]:
        w = (torch.randn(n, k, generator=gen) * 0.7).to(src_dtype)
        q, s = qk.quantize_weight(w.to(cuda_device))
        q_o, s_o, _ = O.quantize(w.float().numpy())
        np.testing.assert_array_equal(q.cpu().numpy(), q_o)
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_o.view(np.uint32))


def test_quantiser_reports_non_finite_weights(cuda_device):
    w = torch.ones(4, 40, device=cuda_device)
    w[2, 7] = float("nan")
    with pytest.raises(ValueError, match="non-finite"):
        qk.quantize_weight(w)
    w[2, 7] = float("inf")
    with pytest.raises(ValueError, match="non-finite"):
        qk.quantize_weight(w)


@pytest.mark.parametrize("kind", [O.BF16, O.F16, O.F32])
def test_dequantize_matches_oracle_bits(cuda_device, kind):
    gen = torch.Generator().manual_seed(4)
    w = torch.randn(37, 70, generator=gen)
    q_o, s_o, _ = O.quantize(w.numpy())
    out = qk.dequantize_weight(torch.from_numpy(q_o).to(cuda_device), torch.from_numpy(s_o).to(cuda_device),
                               TORCH_OF[kind])
    np.testing.assert_array_equal(_np(out), O.dequantize(q_o, s_o, kind))


# ------------------------------------------------------------------------------- GEMMs
def _rand_problem(m, k, n, seed, *, x_std=1.0, w_std=0.02):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen) * x_std
    w = torch.randn(n, k, generator=gen) * w_std
    q, s, _ = O.quantize(w.numpy())
    return x, q, s


def _check_close(actual: np.ndarray, expected: np.ndarray, v_kind: int):
    exp_r = O.round_kind(expected.astype(np.float32), v_kind)
    err = O.rel_fro(actual, expected)
    assert err <= REL_FRO_TOL, f"relative Frobenius error {err:.3e}"
    # elementwise: within 4 ulp of the compute dtype at the output's magnitude
    ulp = 2.0 ** -7 if v_kind == O.BF16 else 2.0 ** -10
    scale = np.maximum(np.abs(exp_r), np.abs(expected).max() * 1e-3 + 1e-30)
    assert np.all(np.abs(actual - expected) <= 4 * ulp * scale + 1e-6), float(np.max(np.abs(actual - expected) / scale))


SHAPES = [
    (6, 70, 37),        # reference ragged case: not TMA-describable, plain-load producer
    (1, 64, 8),
    (128, 64, 256),     # exactly one tile
    (200, 320, 300),    # ragged M and N, TMA path
    (257, 1024, 520),
    (64, 3072, 3072),   # small-M, BASELINE width
    (512, 3072, 1024),
]


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("v_kind", [O.BF16, O.F16])
@pytest.mark.parametrize("with_bias", [True, False])
def test_forward_matches_oracle(cuda_device, m, k, n, v_kind, with_bias):
    x, q, s = _rand_problem(m, k, n, seed=m * 7 + k + n)
    bias = (torch.randn(n) * 0.5) if with_bias else None
    dt = TORCH_OF[v_kind]
    y = qk.int8_linear_forward(
        x.to(cuda_device, dt), torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device),
        None if bias is None else bias.to(cuda_device, dt), dt, dt)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert y.dtype == dt and y.shape == (m, n)
    expected = O.gemm_fwd(_np(x.to(dt)), q, s, w_kind=v_kind, v_kind=v_kind,
                          bias=None if bias is None else _np(bias.to(dt)))
    _check_close(_np(y), expected, v_kind)


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("v_kind", [O.BF16, O.F16])
def test_input_gradient_matches_oracle(cuda_device, m, n, k, v_kind):
    gen = torch.Generator().manual_seed(m + 3 * n + k)
    dy = torch.randn(m, n, generator=gen)
    w = torch.randn(n, k, generator=gen) * 0.02
    q, s, _ = O.quantize(w.numpy())
    dt = TORCH_OF[v_kind]
    dx = qk.int8_linear_backward(dy.to(cuda_device, dt), torch.from_numpy(q).to(cuda_device),
                                 torch.from_numpy(s).to(cuda_device), torch.Size((m, k)), dt, dt)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert dx.shape == (m, k) and dx.dtype == dt
    expected = O.gemm_dx(_np(dy.to(dt)), q, s, w_kind=v_kind, v_kind=v_kind)
    _check_close(_np(dx), expected, v_kind)


@pytest.mark.parametrize("w_kind", [O.F32, O.F16])
def test_mixed_weight_dtype_decode_matches_oracle(cuda_device, w_kind):
    """Module dtype differs from the compute dtype (fp32 module under bf16 autocast)."""
    m, k, n = 96, 192, 160
    x, q, s = _rand_problem(m, k, n, seed=11)
    y = qk.int8_linear_forward(x.to(cuda_device, torch.bfloat16), torch.from_numpy(q).to(cuda_device),
                               torch.from_numpy(s).to(cuda_device), None, torch.bfloat16, TORCH_OF[w_kind])
    expected = O.gemm_fwd(_np(x.to(torch.bfloat16)), q, s, w_kind=w_kind, v_kind=O.BF16)
    _check_close(_np(y), expected, O.BF16)
    dy = torch.randn(m, n, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    dx = qk.int8_linear_backward(dy.to(cuda_device), torch.from_numpy(q).to(cuda_device),
                                 torch.from_numpy(s).to(cuda_device), torch.Size((m, k)), torch.float32,
                                 TORCH_OF[w_kind], compute_dtype=torch.bfloat16)
    assert dx.dtype == torch.float32
    expected_dx = O.round_kind(O.gemm_dx(_np(dy), q, s, w_kind=w_kind, v_kind=O.BF16).astype(np.float32), O.BF16)
    # stored as f32 after rounding through bf16: values are bf16-representable
    assert np.array_equal(O.round_bf16(_np(dx)), _np(dx))
    assert O.rel_fro(_np(dx), expected_dx) <= REL_FRO_TOL


@pytest.mark.parametrize("rank", [8, 32, 64, 96])
def test_fused_lora_terms_match_oracle(cuda_device, rank):
    m, k, n = 200, 256, 384
    gen = torch.Generator().manual_seed(rank)
    x = torch.randn(m, k, generator=gen)
    w = torch.randn(n, k, generator=gen) * 0.02
    q, s, _ = O.quantize(w.numpy())
    xa = (torch.randn(m, rank, generator=gen)).to(torch.bfloat16)
    lb = torch.randn(n, rank, generator=gen) * 0.05
    scale = 0.75
    y = qk.int8_linear_forward(x.to(cuda_device, torch.bfloat16), torch.from_numpy(q).to(cuda_device),
                               torch.from_numpy(s).to(cuda_device), None, torch.bfloat16, torch.bfloat16,
                               lora_xa=xa.to(cuda_device), lora_b=lb.to(cuda_device), lora_scale=scale)
    b_eff = O.round_bf16(lb.numpy() * np.float32(scale))
    expected = O.gemm_fwd(_np(x.to(torch.bfloat16)), q, s, w_kind=O.BF16, v_kind=O.BF16, lora_xa=_np(xa),
                          lora_b=b_eff, lora_scale=1.0)
    _check_close(_np(y), expected, O.BF16)
    # grad-input with the adapter term: dx = dy dec(W) + scale * dyb A
    dy = torch.randn(m, n, generator=gen)
    la = torch.randn(rank, k, generator=gen) * 0.05
    dyb = torch.randn(m, rank, generator=gen).to(torch.bfloat16)
    dx = qk.int8_linear_backward(dy.to(cuda_device, torch.bfloat16), torch.from_numpy(q).to(cuda_device),
                                 torch.from_numpy(s).to(cuda_device), torch.Size((m, k)), torch.bfloat16,
                                 torch.bfloat16, lora_dyb=dyb.to(cuda_device), lora_a=la.to(cuda_device),
                                 lora_scale=scale)
    a_eff = O.round_bf16(la.numpy() * np.float32(scale))
    expected_dx = O.gemm_dx(_np(dy.to(torch.bfloat16)), q, s, w_kind=O.BF16, v_kind=O.BF16, lora_dyb=_np(dyb),
                            lora_a=a_eff, lora_scale=1.0)
    _check_close(_np(dx), expected_dx, O.BF16)


def test_zero_inner_dimension_gives_bias(cuda_device):
    q = torch.empty(5, 0, dtype=torch.int8, device=cuda_device)
    s = torch.ones(5, device=cuda_device)
    x = torch.empty(3, 0, dtype=torch.bfloat16, device=cuda_device)
    bias = torch.arange(5, dtype=torch.bfloat16, device=cuda_device)
    y = qk.int8_linear_forward(x, q, s, bias, torch.bfloat16, torch.bfloat16)
    torch.testing.assert_close(y, bias.expand(3, 5), rtol=0, atol=0)
    empty = qk.int8_linear_forward(torch.empty(0, 8, dtype=torch.bfloat16, device=cuda_device),
                                   torch.zeros(4, 8, dtype=torch.int8, device=cuda_device),
                                   torch.ones(4, device=cuda_device), None, torch.bfloat16, torch.bfloat16)
    assert empty.shape == (0, 4)


@pytest.mark.parametrize("m,k,n", [(4096, 3072, 3072), (4608, 3072, 12288), (4608, 12288, 3072)])
def test_full_size_against_fp32_matmul(cuda_device, m, k, n):
    """BASELINE sizes: fp32 cuBLAS on the oracle-decoded weight is the reference here
    (the fp64 oracle is too slow at this size); TF32 is disabled for the reference."""
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    w = torch.randn(n, k, generator=gen) * 0.02
    q, s, _ = O.quantize(w.numpy())
    dec = torch.from_numpy(O.dequantize(q, s, O.BF16)).to(cuda_device)
    xd = x.to(cuda_device)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    y = qk.int8_linear_forward(xd, qd, sd, None, torch.bfloat16, torch.bfloat16)
    ref = xd.float() @ dec.t()
    assert O.rel_fro(_np(y), _np(ref)) <= REL_FRO_TOL
    dy = torch.randn(m, n, generator=gen).to(torch.bfloat16).to(cuda_device)
    dx = qk.int8_linear_backward(dy, qd, sd, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
    ref_dx = dy.float() @ dec
    assert O.rel_fro(_np(dx), _np(ref_dx)) <= REL_FRO_TOL
    torch.cuda.synchronize()
    _status_ok(cuda_device)


SMALL_M = [
    (2, 3072, 18432),    # per-block adaLN modulation: batch rows only
    (16, 3072, 3072),
    (128, 3072, 3072),
    (1, 12288, 3072),
    (64, 1024, 520),     # ragged N
]


@pytest.mark.parametrize("m,k,n", SMALL_M)
def test_small_m_split_k_forward_and_input_gradient(cuda_device, m, k, n):
    """Small-M problems split the reduction across CTAs (f32 partials in a workspace,
    reduced in fixed order by the last split of each tile)."""
    size = ctypes.c_size_t()
    _lib.check(_lib.library().moss_w8a16_gemm_workspace_bytes(m, n, k, ctypes.byref(size)), "workspace")
    assert size.value > 0 or m > 32
    x, q, s = _rand_problem(m, k, n, seed=m + k + n)
    bias = torch.randn(n) * 0.5
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    y = qk.int8_linear_forward(x.to(cuda_device, torch.bfloat16), qd, sd, bias.to(cuda_device, torch.bfloat16),
                               torch.bfloat16, torch.bfloat16)
    y2 = qk.int8_linear_forward(x.to(cuda_device, torch.bfloat16), qd, sd, bias.to(cuda_device, torch.bfloat16),
                                torch.bfloat16, torch.bfloat16)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert torch.equal(y, y2), "split-K reduction must be deterministic"
    expected = O.gemm_fwd(_np(x.to(torch.bfloat16)), q, s, w_kind=O.BF16, v_kind=O.BF16,
                          bias=_np(bias.to(torch.bfloat16)))
    _check_close(_np(y), expected, O.BF16)
    dy = torch.randn(m, n, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    dx = qk.int8_linear_backward(dy.to(cuda_device), qd, sd, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _check_close(_np(dx), O.gemm_dx(_np(dy), q, s, w_kind=O.BF16, v_kind=O.BF16), O.BF16)


def test_split_k_without_workspace_matches(cuda_device):
    """With no workspace the same problem runs unsplit: same values up to f32 summation order."""
    m, k, n = 8, 3072, 3072
    x, q, s = _rand_problem(m, k, n, seed=21)
    xd = x.to(cuda_device, torch.bfloat16)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    y_split = qk.int8_linear_forward(xd, qd, sd, None, torch.bfloat16, torch.bfloat16)
    y_plain = torch.empty_like(y_split)
    rc = _lib.library().moss_w8a16_gemm_fwd(
        xd.data_ptr(), 1, m, k, qd.data_ptr(), sd.data_ptr(), 1, n, None, 0, None, None, 0, 0, 1.0,
        y_plain.data_ptr(), 1, None, 0, qk.status_buffer(cuda_device).data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gemm")
    torch.cuda.synchronize()
    assert O.rel_fro(_np(y_split), _np(y_plain)) < 2e-3


# ------------------------------------------------------------------ CTA-pair kernel: last-round split
# Shapes whose last round of 256 x 256 tiles leaves SM pairs idle (148 SMs = 74 pairs). The
# reduction lengths are short so the scalar fp64 oracle finishes in seconds.
PAIR_TAIL_FWD = [
    (768, 1088, 6400, 0),      # 75 tiles: 1 left over, split 9 ways = one load step per unit
    (1000, 1088, 4800, 0),     # ragged M and N (76 tiles), 17 k-blocks: the last step holds one
    (768, 1088, 6400, 32),     # fused LoRA term: its k-block lands in the last split
]


def _workspace_bytes(m, n_out, k_red):
    size = ctypes.c_size_t()
    _lib.check(_lib.library().moss_w8a16_gemm_workspace_bytes(m, n_out, k_red, ctypes.byref(size)), "workspace")
    return size.value


def _skip_unless_148_sms(device):
    if torch.cuda.get_device_properties(device).multi_processor_count != 148:
        pytest.skip("the split plans of these shapes assume 148 SMs")


@pytest.mark.parametrize("m,k,n,rank", PAIR_TAIL_FWD)
def test_pair_last_round_split_forward_matches_oracle(cuda_device, m, k, n, rank):
    """The tiles of the last round are split along K: f32 partials in the workspace, reduced
    in split order by the last unit of each 32-row slice. Deterministic, within the oracle
    bound, and equal to the unsplit kernel (no workspace) up to f32 summation order."""
    _skip_unless_148_sms(cuda_device)
    assert _workspace_bytes(m, n, k) > 0
    x, q, s = _rand_problem(m, k, n, seed=m + 3 * k + n)
    gen = torch.Generator().manual_seed(rank + 5)
    bias = torch.randn(n, generator=gen) * 0.5
    xd = x.to(cuda_device, torch.bfloat16)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    bd = bias.to(cuda_device, torch.bfloat16)
    lora, extra = {}, {}
    if rank:
        xa = torch.randn(m, rank, generator=gen).to(torch.bfloat16)
        lb = torch.randn(n, rank, generator=gen) * 0.05
        lora = dict(lora_xa=xa.to(cuda_device), lora_b=lb.to(cuda_device), lora_scale=0.5)
        extra = dict(lora_xa=_np(xa), lora_b=O.round_bf16(lb.numpy() * np.float32(0.5)), lora_scale=1.0)
    y = qk.int8_linear_forward(xd, qd, sd, bd, torch.bfloat16, torch.bfloat16, **lora)
    y2 = qk.int8_linear_forward(xd, qd, sd, bd, torch.bfloat16, torch.bfloat16, **lora)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert torch.equal(y, y2), "the split reduction must be deterministic"
    expected = O.gemm_fwd(_np(x.to(torch.bfloat16)), q, s, w_kind=O.BF16, v_kind=O.BF16,
                          bias=_np(bias.to(torch.bfloat16)), **extra)
    _check_close(_np(y), expected, O.BF16)
    if not rank:
        y_whole = torch.empty_like(y)
        rc = _lib.library().moss_w8a16_gemm_fwd(
            xd.data_ptr(), 1, m, k, qd.data_ptr(), sd.data_ptr(), 1, n, bd.data_ptr(), 1, None, None, 0, 0, 1.0,
            y_whole.data_ptr(), 1, None, 0, qk.status_buffer(cuda_device).data_ptr(),
            torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "gemm")
        torch.cuda.synchronize()
        assert O.rel_fro(_np(y), _np(y_whole)) < 1e-3
        assert (y == y_whole).float().mean().item() > 0.9


def test_pair_last_round_split_grad_input_matches_oracle(cuda_device):
    """Grad-input whose [768, 6400] output is 75 tiles: the last one is split 9 ways."""
    _skip_unless_148_sms(cuda_device)
    m, k, n = 768, 6400, 1088
    assert _workspace_bytes(m, k, n) > 0
    _, q, s = _rand_problem(1, k, n, seed=31)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    dy = torch.randn(m, n, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
    dx = qk.int8_linear_backward(dy.to(cuda_device), qd, sd, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
    dx2 = qk.int8_linear_backward(dy.to(cuda_device), qd, sd, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert torch.equal(dx, dx2)
    _check_close(_np(dx), O.gemm_dx(_np(dy), q, s, w_kind=O.BF16, v_kind=O.BF16), O.BF16)


def test_pair_last_round_split_f16_f32_output_and_lora_grad_input(cuda_device):
    """The split path's reduction kernel with an f16 compute type, with an f32 output buffer
    after the generic decode (f32 module dtype), and a grad-input whose LoRA block lands in
    the last split. 768 x 6400 outputs are 75 tiles: the last one is split 9 ways."""
    _skip_unless_148_sms(cuda_device)
    m, k, n = 768, 1088, 6400
    x, q, s = _rand_problem(m, k, n, seed=51)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    gen = torch.Generator().manual_seed(52)
    bias = torch.randn(n, generator=gen) * 0.5
    # f16 compute
    y16 = qk.int8_linear_forward(x.to(cuda_device, torch.float16), qd, sd, bias.to(cuda_device, torch.float16),
                                 torch.float16, torch.float16)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _check_close(_np(y16), O.gemm_fwd(_np(x.to(torch.float16)), q, s, w_kind=O.F16, v_kind=O.F16,
                                      bias=_np(bias.to(torch.float16))), O.F16)
    # f32 output, f32 module dtype (generic decode), through the C ABI with the workspace
    xd = x.to(cuda_device, torch.bfloat16)
    y32 = torch.empty(m, n, dtype=torch.float32, device=cuda_device)
    owner, ws, ws_bytes = qk._workspace(m, n, k, cuda_device)
    assert ws_bytes > 0
    rc = _lib.library().moss_w8a16_gemm_fwd(
        xd.data_ptr(), 1, m, k, qd.data_ptr(), sd.data_ptr(), 2, n, None, 0, None, None, 0, 0, 1.0,
        y32.data_ptr(), 2, ws, ws_bytes, qk.status_buffer(cuda_device).data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gemm")
    torch.cuda.synchronize()
    del owner
    _status_ok(cuda_device)
    _check_close(y32.cpu().numpy(), O.gemm_fwd(_np(xd), q, s, w_kind=O.F32, v_kind=O.BF16), O.BF16)
    # grad-input [768, 6400] with the adapter term: the LoRA block is the last split's
    md, kd, nd = 768, 6400, 1088
    _, q2, s2 = _rand_problem(1, kd, nd, seed=53)
    q2d, s2d = torch.from_numpy(q2).to(cuda_device), torch.from_numpy(s2).to(cuda_device)
    assert _workspace_bytes(md, kd, nd) > 0
    rank, scale = 32, 0.5
    dy = torch.randn(md, nd, generator=gen).to(torch.bfloat16)
    dyb = torch.randn(md, rank, generator=gen).to(torch.bfloat16)
    la = torch.randn(rank, kd, generator=gen) * 0.05
    dx = qk.int8_linear_backward(dy.to(cuda_device), q2d, s2d, torch.Size((md, kd)), torch.bfloat16, torch.bfloat16,
                                 lora_dyb=dyb.to(cuda_device), lora_a=la.to(cuda_device), lora_scale=scale)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    a_eff = O.round_bf16(la.numpy() * np.float32(scale))
    expected = O.gemm_dx(_np(dy), q2, s2, w_kind=O.BF16, v_kind=O.BF16, lora_dyb=_np(dyb), lora_a=a_eff,
                         lora_scale=1.0)
    _check_close(_np(dx), expected, O.BF16)


def test_pair_last_round_split_long_reduction_against_torch_fp32(cuda_device):
    """The config-5 grad-input of the (3072, 18432) projection at 2048 rows: 144 load steps
    per tile, too long for the scalar oracle, so the reference is a torch fp32 matmul (TF32
    off) on the oracle-decoded weight."""
    _skip_unless_148_sms(cuda_device)
    m, k, n = 2048, 3072, 18432
    assert _workspace_bytes(m, k, n) > 0
    _, q, s = _rand_problem(1, k, n, seed=41)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    dy = torch.randn(m, n, generator=torch.Generator().manual_seed(42)).to(torch.bfloat16).to(cuda_device)
    dx = qk.int8_linear_backward(dy, qd, sd, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
    w = torch.from_numpy(O.dequantize(q, s, O.BF16)).to(cuda_device, torch.float32)
    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = dy.float() @ w
    finally:
        torch.backends.cuda.matmul.allow_tf32 = allow
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _check_close(_np(dx), ref.cpu().double().numpy(), O.BF16)


# ------------------------------------------------------------------ few-row (operand-swapped) kernel
FEW_ROWS = [
    (1, 3072, 3072),     # one token: 24 feature tiles, split over K
    (2, 3072, 18432),    # adaLN modulation rows: 144 tiles, no split
    (16, 12288, 3072),   # MLP down projection, long K split
    (17, 1024, 1280),    # first row past a 16-token tile
    (32, 3072, 3072),
    (33, 2048, 520),     # 64-token tile, ragged features
    (64, 3072, 1536),
    (100, 1024, 3072),   # 128-token tile
    (128, 3072, 1536),
    (200, 2048, 1280),   # 256-token tile, ragged
    (300, 1024, 2560),   # two token tiles, the second ragged
    (512, 1024, 3072),   # too few CTA-pair tiles: operand-swapped kernel with split-K
]


@pytest.mark.parametrize("m,k,n", FEW_ROWS)
@pytest.mark.parametrize("v_dtype", [torch.bfloat16, torch.float16])
def test_few_row_kernel_forward_and_input_gradient(cuda_device, m, k, n, v_dtype):
    """Problems with too few rows for the CTA-pair tiles run the operand-swapped kernel
    (weight as the 128-row MMA operand, up to 256 tokens per tile), split over K when the
    tiles alone cannot occupy the GPU."""
    v_kind = O.BF16 if v_dtype == torch.bfloat16 else O.F16
    x, q, s = _rand_problem(m, k, n, seed=1000 + m + n)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(m)) * 0.5
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    xd = x.to(cuda_device, v_dtype)
    y = qk.int8_linear_forward(xd, qd, sd, bias.to(cuda_device, v_dtype), v_dtype, v_dtype)
    y2 = qk.int8_linear_forward(xd, qd, sd, bias.to(cuda_device, v_dtype), v_dtype, v_dtype)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    assert torch.equal(y, y2), "split-K reduction must be deterministic"
    expected = O.gemm_fwd(_np(x.to(v_dtype)), q, s, w_kind=v_kind, v_kind=v_kind, bias=_np(bias.to(v_dtype)))
    _check_close(_np(y), expected, v_kind)
    dy = torch.randn(m, n, generator=torch.Generator().manual_seed(m + 7)).to(v_dtype)
    dx = qk.int8_linear_backward(dy.to(cuda_device), qd, sd, torch.Size((m, k)), v_dtype, v_dtype)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _check_close(_np(dx), O.gemm_dx(_np(dy), q, s, w_kind=v_kind, v_kind=v_kind), v_kind)


def test_few_row_kernel_mixed_weight_dtype_and_f32_output(cuda_device):
    """Generic decode (module dtype f32, compute bf16) and an f32 output buffer."""
    m, k, n = 8, 1024, 640
    x, q, s = _rand_problem(m, k, n, seed=77)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    xd = x.to(cuda_device, torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.float32, device=cuda_device)
    rc = _lib.library().moss_w8a16_gemm_fwd(
        xd.data_ptr(), 1, m, k, qd.data_ptr(), sd.data_ptr(), 2, n, None, 0, None, None, 0, 0, 1.0,
        y.data_ptr(), 2, None, 0, qk.status_buffer(cuda_device).data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gemm")
    torch.cuda.synchronize()
    expected = O.gemm_fwd(_np(x.to(torch.bfloat16)), q, s, w_kind=O.F32, v_kind=O.BF16)
    _check_close(y.cpu().numpy(), expected, O.BF16)
