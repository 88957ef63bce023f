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


FULL_TENSORS = ["bb.lm_head.weight", "bb.blk.7.ffn_down.weight", "bb.blk.2.attn_output.weight", "dd.in_proj.weight",
                "dd.blk.3.ffn_down.weight"]


@pytest.fixture(scope="module")
def full_gen(pkg):
    import os
    d = os.environ.get("BZB_MODEL_DIR", "/tmp/bzb_models")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "breeze_full_nc32_q8_0_seed0_eosoff.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        pkg.synth_model(tmp, preset="full", nc=32, quant="q8_0", seed=0, eos_off=True, depth_top_k=1)
        os.replace(tmp, path)
    import breeze_oracle as bo
    g = pkg.GeneratorHandle(path, 0)
    yield g, bo.Model(path)
    g.close()


@pytest.mark.parametrize("tensor", FULL_TENSORS)
@pytest.mark.parametrize("rows", [1, 64, 256])
def test_noalloc_gemm_full_size_fits_and_allocates_nothing(full_gen, tensor, rows, monkeypatch):
    """The full model's resident unfused matrices (K up to 8192, the 2052-row LM head) at 1 to
    256 rows fit the fixed scratch: results equal an independent f16-operand product, and the
    device's free memory does not move across two calls (the first call on a device only looks
    up the scratch address). BZB_GEMV_SPLITS, which other paths honour, does not change the plan."""
    import torch
    gen, m = full_gen
    if rows == 64:
        monkeypatch.setenv("BZB_GEMV_SPLITS", "8")
    w = m.w(tensor)
    M, K = w.shape
    x = np.random.default_rng(rows).standard_normal((rows, K)).astype(np.float32)
    x16 = x.astype(np.float16).astype(np.float64)
    w16 = w.astype(np.float16).astype(np.float64)
    ref = x16 @ w16.T
    scale = np.abs(x16) @ np.abs(w16).T + 1e-6
    xd = torch.from_numpy(x).to("cuda", torch.float16)
    yd = torch.zeros((rows, M), dtype=torch.float32, device="cuda")
    gen.gemm_noalloc(tensor, rows, xd.data_ptr(), K, yd.data_ptr(), M)  # first call on this device
    gen.sync()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        yd.zero_()
        torch.cuda.synchronize()
        gen.gemm_noalloc(tensor, rows, xd.data_ptr(), K, yd.data_ptr(), M)
        gen.sync()
        y = yd.cpu().numpy().astype(np.float64)
        assert np.max(np.abs(y - ref) / scale) < 1e-5
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
