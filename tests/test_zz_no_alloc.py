"""lb_op_gemm_splitk_scratch (fixed in-library device scratch, no allocation)
against lb_op_gemm, the GEMM entry point it is a variant of, and against a plain
fp32 torch product of the same operands.

Collected last on purpose: it must pass after every other test has run in the
same process, and ``test_fresh_process`` runs the same check in a new
interpreter where the entry point's one-time device setup happens first.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

LB_ERR_CAPACITY = -4
SCRATCH_FLOATS = 1 << 21

# (m, out_features, k, weight kind, act, splits, bias, extra output columns);
# weight kind 0 = bf16, 1 = int8 codes, 2 = int8 codes widened to fp16
CASES = [
    (64, 1536, 6144, 1, 0, 4, True, 0),
    (200, 6144, 1536, 0, 1, 2, True, 128),
    (1, 1536, 1536, 1, 1, 3, False, 0),
    (130, 2048, 3072, 0, 0, 1, False, 0),
    (96, 1536, 3072, 2, 1, 2, True, 0),
]


def _operands(m, o, k, int8, bias, seed):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.float16 if int8 else torch.bfloat16).to(dev)
    if int8:
        w = torch.randint(-127, 128, (o, k), generator=g, dtype=torch.int8).to(dev)
        if int8 == 2:
            w = w.to(torch.float16)
        sc = (torch.rand(o, generator=g) * 1e-3 + 1e-4).to(torch.float16).to(dev)
    else:
        w = (torch.randn(o, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        sc = None
    b = (torch.randn(o, generator=g) * 0.1).to(dev) if bias else None
    return x, w, sc, b


def check_against_lb_op_gemm(lib) -> None:
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, (m, o, k, int8, act, splits, bias, pad) in enumerate(CASES):
        x, w, sc, b = _operands(m, o, k, int8, bias, seed=1000 + i)
        sptr = sc.data_ptr() if sc is not None else None
        bptr = b.data_ptr() if b is not None else None
        ref = torch.zeros(m, o, dtype=torch.bfloat16, device="cuda")
        rc = lib.lb_op_gemm(x.data_ptr(), k, m, w.data_ptr(), int(int8), sptr, bptr, o, k,
                            ref.data_ptr(), o, 0, act, 1, status.data_ptr(), stream)
        assert rc == 0
        ref = ref.float()
        tol = 1.6e-2 * ref.abs() + 4e-3 * ref.abs().max()
        ld = o + pad
        for call in range(2):  # the second call must not see the first call's partial sums
            out = torch.full((m, ld), float("nan"), dtype=torch.bfloat16, device="cuda")
            rc = lib.lb_op_gemm_splitk_scratch(x.data_ptr(), k, m, w.data_ptr(), int(int8), sptr, bptr,
                                               o, k, out.data_ptr(), ld, act, splits,
                                               status.data_ptr(), stream)
            assert rc == 0, (i, call, rc)
            torch.cuda.synchronize()
            assert status.item() == 0, (i, call, status.item())
            got = out[:, :o].float()
            err = (got - ref).abs()
            assert bool((err <= tol).all()), (i, call, float(err.max()), float(ref.abs().max()))
            if pad:
                assert bool(torch.isnan(out[:, o:].float()).all()), "wrote past out_features"


@pytest.fixture(scope="module")
def lib(pkg):
    from gemma4_omni_b200 import _lib
    return _lib.load()


def test_matches_lb_op_gemm_twice_in_a_row(lib):
    check_against_lb_op_gemm(lib)


def test_matches_a_plain_fp32_torch_product(lib):
    """The scratch entry point against the arithmetic itself: x . (scale * W)^T + bias
    in fp32 torch, SiLU of the bf16-rounded linear output, bf16 result."""
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, (m, o, k, int8, act, splits, bias, _) in enumerate(CASES):
        x, w, sc, b = _operands(m, o, k, int8, bias, seed=2000 + i)
        w_ref = w.float() * sc.float()[:, None] if sc is not None else w.float()
        ref = x.float() @ w_ref.t()
        if b is not None:
            ref = ref + b
        if act:
            ref = torch.nn.functional.silu(ref.to(torch.bfloat16).float())
        out = torch.zeros(m, o, dtype=torch.bfloat16, device="cuda")
        rc = lib.lb_op_gemm_splitk_scratch(x.data_ptr(), k, m, w.data_ptr(), int(int8),
                                           sc.data_ptr() if sc is not None else None,
                                           b.data_ptr() if b is not None else None, o, k, out.data_ptr(), o,
                                           act, splits, status.data_ptr(), stream)
        torch.cuda.synchronize()
        assert rc == 0 and status.item() == 0, (i, rc, status.item())
        # bf16 output: one rounding (2^-8 relative), plus a possible one-ulp flip of
        # the pre-SiLU rounding under a different fp32 summation order
        torch.testing.assert_close(out.float(), ref, rtol=1.6e-2, atol=4e-3 * ref.abs().max().item())


def test_rejects_sizes_beyond_scratch(lib):
    x = torch.zeros(8, 1536, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(8, 1536, dtype=torch.bfloat16, device="cuda")
    m = SCRATCH_FLOATS // 1536 + 1  # m * out_features just above the scratch size
    rc = lib.lb_op_gemm_splitk_scratch(x.data_ptr(), 1536, m, x.data_ptr(), 0, None, None, 1536, 1536,
                                       out.data_ptr(), 1536, 0, 2, None,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == LB_ERR_CAPACITY


def test_rejects_bad_shapes_strides_and_alignment(lib):
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(8, 512, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(512, 512, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(8, 512, dtype=torch.bfloat16, device="cuda")

    def call(xp=None, x_ld=512, o=256, k=256, outp=None, ld_out=256):
        return lib.lb_op_gemm_splitk_scratch(xp or x.data_ptr(), x_ld, 8, w.data_ptr(), 0, None, None, o, k,
                                             outp or out.data_ptr(), ld_out, 0, 2, None, stream)

    assert call(o=192, ld_out=192) == -1                # out_features not a multiple of 128
    assert call(k=96) == -1                             # k not a multiple of 64
    assert call(ld_out=128) == -1                       # ld_out < out_features
    assert call(outp=out.data_ptr() + 2) == -1          # out not 16-byte aligned
    assert call(x_ld=128) == -1                         # x_ld < k: rows would overlap
    assert call(xp=x.data_ptr() + 2) == -1              # x not 16-byte aligned
    assert call() == 0
    torch.cuda.synchronize()


def test_splits_beyond_k_blocks_are_clamped(lib):
    """splits > k/64 runs with one K block per split; the result still matches lb_op_gemm."""
    stream = torch.cuda.current_stream().cuda_stream
    m, o, k = 40, 1536, 512  # 8 K blocks
    x, w, _, b = _operands(m, o, k, 0, True, seed=77)
    ref = torch.zeros(m, o, dtype=torch.bfloat16, device="cuda")
    assert lib.lb_op_gemm(x.data_ptr(), k, m, w.data_ptr(), 0, None, b.data_ptr(), o, k, ref.data_ptr(), o, 0, 0,
                          1, None, stream) == 0
    out = torch.zeros(m, o, dtype=torch.bfloat16, device="cuda")
    assert lib.lb_op_gemm_splitk_scratch(x.data_ptr(), k, m, w.data_ptr(), 0, None, b.data_ptr(), o, k,
                                         out.data_ptr(), o, 0, 64, None, stream) == 0
    torch.cuda.synchronize()
    ref = ref.float()
    assert bool(((out.float() - ref).abs() <= 1.6e-2 * ref.abs() + 4e-3 * ref.abs().max()).all())


def test_fresh_process():
    res = subprocess.run([sys.executable, str(Path(__file__).resolve())], capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0 and "no-alloc ok" in res.stdout, res.stdout + res.stderr


if __name__ == "__main__":
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from conftest import load_package

    load_package()
    from gemma4_omni_b200 import _lib

    check_against_lb_op_gemm(_lib.load())
    print("no-alloc ok")
