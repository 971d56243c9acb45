"""Host-side argument checks of the Python bindings: shape and type errors are raised before any
device call, so they hold on a CPU-only host."""

import pytest


def test_gemm_mx_shape_checks(ptxstd_lib):
    import torch

    import ptxstd
    a = torch.zeros((256, 128), dtype=torch.uint8)
    sfa = torch.zeros(256 * 128 // 32, dtype=torch.uint8)
    with pytest.raises(ValueError, match="K mismatch"):
        ptxstd.gemm_mx(a, "e2m3", sfa, torch.zeros((256, 64), dtype=torch.uint8), "e2m3", sfa)
    with pytest.raises(ValueError, match="one UE8M0 per 32"):
        ptxstd.gemm_mx(a, "e2m3", sfa[:-1], a, "e2m3", sfa)
    with pytest.raises(ValueError, match="unknown MX element type"):
        ptxstd.gemm_mx(a, "e9m9", sfa, a, "e2m3", sfa)
    with pytest.raises(ValueError, match="unknown MX element type"):
        ptxstd.gemm_mx(a, 2, sfa, a, "e2m3", sfa)   # 2 is not a tcgen05 element-type code


def test_quantize_mx_input_checks(ptxstd_lib):
    import torch

    import ptxstd
    with pytest.raises(TypeError):
        ptxstd.quantize_mx(torch.zeros((128, 128), dtype=torch.float32), "e4m3")
    with pytest.raises(TypeError):
        ptxstd.quantize_mx(torch.zeros(128, dtype=torch.bfloat16), "e4m3")


def test_cp_unpack_shape_checks(ptxstd_lib):
    import torch

    import ptxstd
    with pytest.raises(ValueError):
        ptxstd.tcgen05_cp_unpack(torch.zeros((100, 32), dtype=torch.uint8), "e2m3")
    with pytest.raises(ValueError):
        ptxstd.tcgen05_cp_unpack(torch.zeros((128, 16), dtype=torch.uint8), "e2m1")
    with pytest.raises(ValueError, match="FP6"):
        ptxstd.tcgen05_cp_unpack(torch.zeros((128, 32), dtype=torch.uint8), "e4m3")


def test_mx_type_names(ptxstd_lib):
    import ptxstd
    from ptxstd import kernels
    assert kernels.MX_TYPES == {"e4m3": 0, "e5m2": 1, "e2m3": 3, "e3m2": 4, "e2m1": 5}
    assert (ptxstd.MX_E4M3, ptxstd.MX_E5M2, ptxstd.MX_E2M3, ptxstd.MX_E3M2,
            ptxstd.MX_E2M1) == (0, 1, 3, 4, 5)


def test_gemm_schedule_setting(ptxstd_lib):
    """The tile-schedule setting round-trips and rejects unknown values (no device needed)."""
    import ptxstd
    assert ptxstd.get_gemm_schedule() == ptxstd.SCHEDULE_PERSISTENT
    try:
        ptxstd.set_gemm_schedule(ptxstd.SCHEDULE_DYNAMIC)
        assert ptxstd.get_gemm_schedule() == ptxstd.SCHEDULE_DYNAMIC
        with pytest.raises(ptxstd.PtxStdError):
            ptxstd.set_gemm_schedule(2)
        assert ptxstd.get_gemm_schedule() == ptxstd.SCHEDULE_DYNAMIC
    finally:
        ptxstd.set_gemm_schedule(ptxstd.SCHEDULE_PERSISTENT)
