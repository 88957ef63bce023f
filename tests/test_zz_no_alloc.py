"""The allocation-free dequant-GEMM entry point (bzb_generator_gemm_noalloc) against the
existing one (bzb_generator_debug_gemv) on the same weights and inputs, two calls in a row.
Collected last; passes alone and after the other GPU tests (needs a B200)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TENSORS = ["bb.blk.1.ffn_down.weight", "bb.lm_head.weight", "dd.blk.0.attn_output.weight", "dd.in_proj.weight"]


@pytest.fixture(scope="module")
def gen(pkg, tiny_model):
    g = pkg.GeneratorHandle(tiny_model, 0)
    yield g
    g.close()


def _check(y, ref, x, w):
    # both paths use f16 activations, f16(q*d) weights and f32 accumulation; they differ only in
    # summation order, bounded relative to the sum of absolute products
    scale = np.abs(x.astype(np.float16).astype(np.float64)) @ np.abs(w.astype(np.float16).astype(np.float64)).T + 1e-6
    assert np.max(np.abs(y - ref) / scale) < 1e-5


@pytest.mark.parametrize("tensor", TENSORS)
@pytest.mark.parametrize("rows", [1, 37, 256])
def test_noalloc_gemm_matches_existing_entry_point_twice(gen, tiny_oracle, tensor, rows):
    import torch
    w = tiny_oracle.w(tensor)
    M, K = w.shape
    ldx, ldy = K + 8, M + 3
    rng = np.random.default_rng(rows * 7 + len(tensor))
    for call in range(2):
        x = rng.standard_normal((rows, K)).astype(np.float32)
        ref = gen.debug_gemv(tensor, x, M)
        xd = torch.zeros((rows, ldx), dtype=torch.float16, device="cuda")
        xd[:, :K] = torch.from_numpy(x).to("cuda", torch.float16)
        yd = torch.full((rows, ldy), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        gen.gemm_noalloc(tensor, rows, xd.data_ptr(), ldx, yd.data_ptr(), ldy)
        gen.sync()
        y = yd[:, :M].cpu().numpy()
        assert np.isfinite(y).all(), (tensor, rows, call)
        assert torch.isnan(yd[:, M:]).all(), "wrote past the output rows"
        _check(y, ref, x, w)


def test_noalloc_gemm_on_a_caller_stream(gen, tiny_oracle):
    import torch
    tensor = "bb.blk.0.attn_output.weight"
    w = tiny_oracle.w(tensor)
    M, K = w.shape
    x = np.random.default_rng(1).standard_normal((16, K)).astype(np.float32)
    ref = gen.debug_gemv(tensor, x, M)
    s = torch.cuda.Stream()
    xd = torch.from_numpy(x).to("cuda", torch.float16)
    yd = torch.zeros((16, M), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(2):
        gen.gemm_noalloc(tensor, 16, xd.data_ptr(), K, yd.data_ptr(), M, s.cuda_stream)
        s.synchronize()
        _check(yd.cpu().numpy(), ref, x, w)


def test_noalloc_gemm_rejects_bad_inputs(gen, tiny_oracle):
    import torch
    tensor = "bb.lm_head.weight"
    M, K = tiny_oracle.w(tensor).shape
    xd = torch.zeros((300, K), dtype=torch.float16, device="cuda")
    yd = torch.zeros((300, M), dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="rows"):
        gen.gemm_noalloc(tensor, 257, xd.data_ptr(), K, yd.data_ptr(), M)
    with pytest.raises(RuntimeError, match="rows"):
        gen.gemm_noalloc(tensor, 0, xd.data_ptr(), K, yd.data_ptr(), M)
    with pytest.raises(RuntimeError, match="resident"):
        gen.gemm_noalloc("bb.blk.0.attn_q.weight", 4, xd.data_ptr(), K, yd.data_ptr(), M)
    with pytest.raises(RuntimeError, match="stride"):
        gen.gemm_noalloc(tensor, 4, xd.data_ptr(), K - 2, yd.data_ptr(), M)
    with pytest.raises(RuntimeError, match="output stride"):
        gen.gemm_noalloc(tensor, 4, xd.data_ptr(), K, yd.data_ptr(), M - 1)
