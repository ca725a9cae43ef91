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


def test_gemm_rejects_bad_strides_and_alignment(lib):
    s = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(8, 256, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(256, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(8, 256, device="cuda")
    args = lambda xp, x_ld, ld_out, o=256, mode=1: (xp, x_ld, 8, w.data_ptr(), 0, None, None, o, 128,
                                                     out.data_ptr(), ld_out, mode, 0, 1, None, s)
    assert lib.lb_op_gemm(*args(x.data_ptr(), 64, 256)) == -1           # x_ld < k: rows would overlap
    assert lib.lb_op_gemm(*args(x.data_ptr() + 2, 256, 256)) == -1      # x not 16-byte aligned
    assert lib.lb_op_gemm(*args(x.data_ptr(), 256, 128)) == -1          # ld_out < out_features
    assert lib.lb_op_gemm(*args(x.data_ptr(), 256, 256, o=192)) == -1   # out_features % 128
    bounds = torch.tensor([-1.0, 1.0])
    rc = lib.lb_op_gemm_clipped(x.data_ptr(), 256, 8, 0, w.data_ptr(), 0, None, None, 256, 128,
                                out.data_ptr(), 256, 2, 0, 2, 1, bounds.data_ptr(), None, None, None, s)
    assert rc == -1  # atomically accumulated partial sums cannot be clamped
    rc = lib.lb_op_gemm_clipped(x.data_ptr(), 256, 8, 0, w.data_ptr(), 0, None, None, 256, 128,
                                out.data_ptr(), 256, 1, 0, 2, 1, bounds.data_ptr(), None, None, None, s)
    assert rc == -1  # a split-K reduction with a finish pass needs its workspace
    rc = lib.lb_op_gemm_clipped(x.data_ptr(), 128, 8, 4, w.data_ptr(), 0, None, None, 384, 128,
                                out.data_ptr(), 384, 1, 0, 1, 3, None, None, None, None, s)
    assert rc == -1  # a part's activation block (4 rows apart) shorter than m


def run_clipped(lib, M, O, K, int8, mode, act, parts, x_part_rows, seed, bias=True, splits=1, calls=1):
    """lb_op_gemm_clipped vs torch: per-part output clamp, SiLU, next-input clamp;
    splits > 1 reduces through the workspace and a finish pass (workspace zero
    on entry, checked zero again after every call)."""
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    dt = torch.float16 if int8 else torch.bfloat16
    rows = (parts - 1) * x_part_rows + M if x_part_rows else M
    x = (torch.randn(rows, K, generator=g) * 0.5).to(dt).to(dev)
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
    # bounds that bind on a few per cent of the outputs, different per part and per side
    scale = 0.02 * K ** 0.5 if not int8 else (w_ref.float().std() * K ** 0.5).item()
    ob = torch.tensor([[-(1.2 + 0.3 * j) * scale, (1.0 + 0.4 * j) * scale] for j in range(parts)],
                      dtype=torch.float32)
    pb = torch.tensor([-0.05, 0.6 * scale]) if act else None
    po = O // parts
    ref = torch.empty(M, O, device=dev)
    hits = 0
    for j in range(parts):
        xj = x[j * x_part_rows:j * x_part_rows + M] if x_part_rows else x[:M]
        yj = xj.float() @ w_ref[j * po:(j + 1) * po].t()
        if bias:
            yj = yj + b[j * po:(j + 1) * po]
        ref[:, j * po:(j + 1) * po] = torch.clamp(yj, float(ob[j, 0]), float(ob[j, 1]))
        hits += int(((yj < float(ob[j, 0])) | (yj > float(ob[j, 1]))).sum())
    if act:
        ref = torch.clamp(torch.nn.functional.silu(ref.to(torch.bfloat16).float()), float(pb[0]), float(pb[1]))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    acc = torch.zeros(M, O, device=dev) if splits > 1 else None
    for _ in range(calls):
        out = torch.zeros(M, O, dtype=torch.bfloat16 if mode == 0 else torch.float32, device=dev)
        rc = lib.lb_op_gemm_clipped(x.data_ptr(), K, M, x_part_rows, wptr, int8, sptr,
                                    b.data_ptr() if bias else None, O, K, out.data_ptr(), O, mode, act, splits,
                                    parts, ob.reshape(-1).contiguous().data_ptr(),
                                    pb.data_ptr() if pb is not None else None,
                                    acc.data_ptr() if acc is not None else None, status.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0 and status.item() == 0
        if splits > 1:
            assert acc.abs().max().item() == 0, "workspace not left zero"
    # the bounds must bind somewhere, or the check is vacuous
    assert hits >= max(1, M * O // 1000), hits
    return out.float(), ref


@pytest.mark.parametrize("M", [2, 96, 600, 2048])
@pytest.mark.parametrize("int8", [0, 1, 2])
@pytest.mark.parametrize("mode,act", [(1, 0), (0, 0), (0, 1)])
def test_gemm_clip_bounds_match_torch(lib, M, int8, mode, act):
    """Finite output clamps (and, with SiLU, the next input's clamp) in the epilogue."""
    out, ref = run_clipped(lib, M, 1536, 1536, int8, mode, act, 1, 0, seed=300 + M + 7 * int8)
    if mode == 1:
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())
    else:
        torch.testing.assert_close(out, ref, rtol=1.6e-2, atol=1e-3)


@pytest.mark.parametrize("M", [2, 96, 2048])
@pytest.mark.parametrize("int8", [0, 1, 2])
@pytest.mark.parametrize("x_parts", [False, True])
def test_gemm_stacked_qkv_parts_match_torch(lib, M, int8, x_parts):
    """The fused Q/K/V form: three stacked linears with their own output clamps,
    and (x_parts) their own activation blocks (per-projection input clamps)."""
    out, ref = run_clipped(lib, M, 3 * 1536, 1536, int8, 0, 0, 3, M + 64 if x_parts else 0,
                           seed=500 + M + int8)
    torch.testing.assert_close(out, ref, rtol=1.6e-2, atol=1e-3)


@pytest.mark.parametrize("M", [2, 40, 300])
@pytest.mark.parametrize("int8", [0, 1, 2])
@pytest.mark.parametrize("mode,act,splits", [(1, 0, 3), (0, 1, 4), (0, 0, 6)])
def test_gemm_split_k_with_finish_pass_matches_torch(lib, M, int8, mode, act, splits):
    """K splits reduced through the workspace, the finish pass applying clamps /
    SiLU; two calls in a row (the workspace is reused)."""
    out, ref = run_clipped(lib, M, 1536, 3072, int8, mode, act, 1, 0, seed=900 + M + int8 + splits,
                           splits=splits, calls=2)
    if mode == 1:
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())
    else:
        torch.testing.assert_close(out, ref, rtol=1.6e-2, atol=1e-3)


@pytest.mark.parametrize("x_parts", [False, True])
def test_gemm_split_k_stacked_parts_match_torch(lib, x_parts):
    out, ref = run_clipped(lib, 24, 3 * 1536, 1536, 1, 0, 0, 3, 64 if x_parts else 0, seed=77, splits=3, calls=2)
    torch.testing.assert_close(out, ref, rtol=1.6e-2, atol=1e-3)
