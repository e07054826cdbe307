"""Host-side planning of the pipelined row-streaming kernel
(objb_pipe_plan_info): the ring budget per caller, the row format of the
MoE down rows, and which x vectors the kernel forms itself.  Pure host
arithmetic: runs without a GPU."""
import math

import pytest

from oracle import oracle as O

SMS = 148  # B200


def _plan(*args, **kw):
    from objeta_b200.quant import pipe_plan_info
    return pipe_plan_info(*args, **kw)


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q5_0, O.IQ3_0, O.FP4_E2M1])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (151936, 2048)])
def test_sweep_shapes_fit_their_ring(fmt, rows, cols):
    """Every configs[1] GEMV takes the pipelined kernel with at least two
    ring slots inside the plain-GEMV budget, and a stage holds at least one
    4-row batch per row group."""
    for moe in (False, True):
        p = _plan(fmt, rows, cols, moe_program=moe)
        assert p["ring_budget"] == (226 if moe else 200) * 1024
        assert p["slots"] >= 2
        assert p["smem_bytes"] <= p["ring_budget"]
        assert p["slots"] * p["slot_bytes"] < p["smem_bytes"] + 1
        assert p["nseg"] * p["ngrp"] <= 15


def test_moe_budget_adds_a_stage_for_wide_rows():
    gemv = _plan(O.Q4_0, 151936, 2048)
    moe = _plan(O.Q4_0, 151936, 2048, moe_program=True)
    assert (gemv["slots"], moe["slots"]) == (2, 3)
    assert gemv["rows_per_stage"] == moe["rows_per_stage"] == gemv["busy_quantum"]


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q5_0, O.IQ3_0])
def test_digit_images_in_kernel_up_to_4096_columns(fmt):
    assert _plan(fmt, 4096, 4096)["x_in_kernel"] == 1
    assert _plan(fmt, 151936, 2048)["x_in_kernel"] == 1
    assert _plan(fmt, 4096, 14336)["x_in_kernel"] == 0


def test_float_quads_in_kernel_except_split_fp4():
    assert _plan(O.FP4_E2M1, 4096, 14336)["x_in_kernel"] == 1
    assert _plan(O.FP4_E2M1, 4096, 4096, split_fp4=True)["x_in_kernel"] == 0


def test_split_fp4_down_rows_keep_every_warp_busy():
    """configs[3] down: O = 4096 rows, so a CTA owns ceil(4096 / 148) -> 28
    rows of each expert.  Two split-FP4 blocks per lane put a 2048-column row
    on one warp and need 60 rows per stage to busy all 15 row groups; one
    block per lane puts it on two warps, 7 row groups, 28 rows."""
    per_cta = math.ceil(4096 / SMS)
    per_cta = (per_cta + 3) // 4 * 4
    two = _plan(O.FP4_E2M1, 4096, 2048, split_fp4=True, blocks_per_lane=2, moe_program=True)
    one = _plan(O.FP4_E2M1, 4096, 2048, split_fp4=True, blocks_per_lane=1, moe_program=True)
    assert per_cta == 28
    assert (two["nseg"], two["busy_quantum"]) == (1, 60) and two["busy_quantum"] > per_cta
    assert (one["nseg"], one["ngrp"], one["busy_quantum"]) == (2, 7, per_cta)


def test_rejects_bad_plans():
    import objeta_b200
    with pytest.raises(objeta_b200.CudaError):
        _plan(O.Q4_0, 16, 33)
    with pytest.raises(objeta_b200.CudaError):
        _plan(O.Q4_0, 16, 64, blocks_per_lane=1)  # one block per lane: split FP4 only
    with pytest.raises(objeta_b200.CudaError):
        _plan(O.Q4_0, 16, 64, split_fp4=True)
