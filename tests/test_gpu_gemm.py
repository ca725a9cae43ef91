"""tcgen05 GEMM (lb_op_gemm) vs a plain PyTorch fp32 reference of the same op."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(pkg):
    from gemma4_omni_b200 import _lib
    return _lib.load()


def run_gemm(lib, M, O, K, int8, mode, act, splits, bias, seed):
    """int8: 0 = bf16 weights, 1 = int8 codes, 2 = the int8 codes widened to fp16."""
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    int8 = int(int8)
    # int8 weights take fp16 activations (the int8 codes widen exactly to fp16)
    x = (torch.randn(M, K, generator=g) * 0.5).to(torch.float16 if int8 else torch.bfloat16).to(dev)
    if int8:
        wq = torch.randint(-127, 128, (O, K), generator=g, dtype=torch.int8).to(dev)
        sc = (torch.rand(O, generator=g) * 1e-3 + 1e-4).to(torch.float16).to(dev)
        w_ref = wq.float() * sc.float()[:, None]
        if int8 == 2:
            wq = wq.to(torch.float16)
        wptr, sptr = wq.data_ptr(), sc.data_ptr()
    else:
        w = (torch.randn(O, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        w_ref, wptr, sptr = w.float(), w.data_ptr(), None
    b = (torch.randn(O, generator=g) * 0.1).to(dev) if bias else None
    ref = x.float() @ w_ref.t()
    if bias:
        ref = ref + b
    if act:
        ref = torch.nn.functional.silu(ref.to(torch.bfloat16).float())
    out = torch.zeros(M, O, dtype=torch.bfloat16 if mode == 0 else torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.lb_op_gemm(x.data_ptr(), K, M, wptr, int8, sptr, b.data_ptr() if bias else None, O, K,
                        out.data_ptr(), O, mode, act, splits, status.data_ptr(),
                        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0 and status.item() == 0
    return out.float(), ref


@pytest.mark.parametrize("M", [1, 2, 31, 64, 200, 300, 2048])
@pytest.mark.parametrize("int8", [0, 1, 2])
def test_gemm_fp32_out_matches_torch(lib, M, int8):
    out, ref = run_gemm(lib, M, 1536, 1536, int8, 1, 0, 1, False, seed=M)
    # fp32 output: only summation order differs from the fp32 reference
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())


# With O = 1536 these token counts select every token-tile width the kernel
# has beyond 256 tokens (144, 160, ..., 256), each with a ragged last tile.
@pytest.mark.parametrize("M", [1537, 1729, 1921, 2113, 2305, 2497, 2689, 2881])
@pytest.mark.parametrize("int8", [0, 1, 2])
def test_gemm_every_token_tile_width(lib, M, int8):
    out, ref = run_gemm(lib, M, 1536, 1536, int8, 1, 0, 1, True, seed=7 + M)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())


@pytest.mark.parametrize("M", [2, 130, 600, 2048])
@pytest.mark.parametrize("int8", [0, 1, 2])
def test_gemm_bf16_silu_bias_matches_torch(lib, M, int8):
    out, ref = run_gemm(lib, M, 6144, 1536, int8, 0, 1, 1, True, seed=100 + M)
    # bf16 output: the result is rounded once (<= 1 ulp = 2^-7 relative) and the
    # pre-SiLU bf16 rounding may flip by one ulp under fp32 summation order
    torch.testing.assert_close(out, ref, rtol=1.6e-2, atol=1e-3)


@pytest.mark.parametrize("M,splits", [(40, 2), (40, 7), (40, 24), (512, 3), (777, 2)])
@pytest.mark.parametrize("int8", [0, 1, 2])
def test_gemm_split_k_atomic_matches_torch(lib, M, splits, int8):
    # split-K partial sums (fp32 atomics) over one token tile (M = 40) and several (M = 512, 777)
    out, ref = run_gemm(lib, M, 1536, 6144, int8, 2, 0, splits, True, seed=splits + M)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())


def test_gemm_rejects_bad_shapes(lib):
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(4, 128, device="cuda")
    rc = lib.lb_op_gemm(x.data_ptr(), 100, 4, x.data_ptr(), 0, None, None, 128, 100, out.data_ptr(), 128,
                        1, 0, 1, None, torch.cuda.current_stream().cuda_stream)
    assert rc == -1  # K not a multiple of 64
