"""Selector preparation on the GPU: bit-exact against the oracle and the reference fixtures."""
import os

import numpy as np
import pytest
import torch

import cvmm_codex_b200.api as C
from cvmm_codex_b200 import ops
from oracle import cvmm_oracle as O

pytestmark = pytest.mark.gpu
SEL = torch.load(os.path.join(os.path.dirname(__file__), "golden", "selector.pt"))


def _check_against_oracle(sel_cpu: torch.Tensor):
    sel = sel_cpu.cuda()
    k = sel.shape[-1]
    raw, ssel, si, oi = O.prepare_sel2(sel_cpu.numpy())
    tok = C.cvmm_prepare_sel2(sel)
    assert tok.raw_sel.dtype == torch.int32 and tok.sel.dtype == torch.int32
    assert tok.sel_index.dtype == torch.int64 and tok.out_index.dtype == torch.int64
    assert tok.raw_sel.shape == sel.shape and tok.sel.shape == sel.shape
    np.testing.assert_array_equal(tok.raw_sel.flatten().cpu().numpy(), raw)
    np.testing.assert_array_equal(tok.sel.flatten().cpu().numpy(), ssel)
    np.testing.assert_array_equal(tok.sel_index.cpu().numpy(), si)
    np.testing.assert_array_equal(tok.out_index.cpu().numpy(), oi)
    rte = C.cvmm_prepare_sel2(sel, route_input=True)
    assert rte.out_index is None
    np.testing.assert_array_equal(rte.sel_index.cpu().numpy(), oi)
    np.testing.assert_array_equal(rte.sel.flatten().cpu().numpy(), ssel)
    del k


@pytest.mark.parametrize("name", sorted(SEL))
def test_selector_fixtures(name):
    c = SEL[name]
    sel = c["sel"]
    tok = C.cvmm_prepare_sel2(sel.cuda())
    # values bit-exact with the reference's cvmm_prepare_sel2 output
    np.testing.assert_array_equal(tok.raw_sel.cpu().numpy(), c["raw_sel"].numpy())
    np.testing.assert_array_equal(tok.sel.cpu().numpy(), c["sorted_sel"].numpy())
    # permutation bit-exact with the stable order
    np.testing.assert_array_equal(tok.out_index.cpu().numpy(), c["stable_index"].numpy())
    np.testing.assert_array_equal(tok.sel_index.cpu().numpy(), c["stable_index"].numpy() // sel.shape[-1])
    offs = ops.expert_offsets(tok.sel, c["n_experts"])
    np.testing.assert_array_equal(offs.cpu().numpy(), c["offsets"].numpy())
    _check_against_oracle(sel)


@pytest.mark.parametrize("R,E,k", [(4096, 8, 2), (65536, 64, 4), (262144, 128, 8), (524288, 128, 64),
                                   (131072, 512, 8), (1 << 20, 1024, 16)])
def test_selector_full_sizes(R, E, k):
    g = torch.Generator().manual_seed(R + E)
    sel = torch.randint(0, E, (R // k, k), generator=g)
    _check_against_oracle(sel)


def test_selector_skewed_and_single_expert():
    g = torch.Generator().manual_seed(7)
    p = torch.arange(1, 129, dtype=torch.float64).pow(-1.1)
    sel = torch.multinomial(p, 32768 * 8, replacement=True, generator=g).view(32768, 8)
    _check_against_oracle(sel)
    _check_against_oracle(torch.full((1000, 4), 3, dtype=torch.int64))


def test_selector_wide_key_range_multi_pass():
    # Keys spread over > 2048 values take more than one radix pass.
    g = torch.Generator().manual_seed(11)
    _check_against_oracle(torch.randint(0, 5000, (3000, 4), generator=g))
    _check_against_oracle(torch.randint(0, 1 << 30, (512, 8), generator=g))
    _check_against_oracle(torch.randint(-1000, 1000, (700, 3), generator=g))


def test_selector_int32_input_and_empty():
    g = torch.Generator().manual_seed(5)
    sel = torch.randint(0, 64, (999, 3), generator=g, dtype=torch.int32)
    _check_against_oracle(sel)
    empty = C.cvmm_prepare_sel2(torch.zeros((0, 4), dtype=torch.int64, device="cuda"))
    assert empty.sel.shape == (0, 4) and empty.sel_index.numel() == 0


def test_expert_offsets_kernel_matches_reference_formula():
    # The reference's own known-answer test (test_cvmm_correctness.py:73-86).
    C.create_kernels()
    for n_experts in (1, 7, 64, 512):
        for total in (1, 13, 1000):
            s = torch.randint(0, n_experts, (total,), device="cuda", dtype=torch.int32).sort().values
            fast = C._cvmm_expert_offsets(s, n_experts)
            old = C.cvmm_expert_offsets_call
            C.cvmm_expert_offsets_call = None
            try:
                ref = C._cvmm_expert_offsets(s, n_experts)
            finally:
                C.cvmm_expert_offsets_call = old
            torch.testing.assert_close(fast.cpu(), ref.cpu(), rtol=0, atol=0)


@pytest.mark.parametrize("R,E", [(64, 8), (4096, 8), (65536, 64), (262144, 128), (524288, 128)])
def test_cuda_default_sort_agrees_with_stable_order(R, E):
    """The reference sorts with CUDA torch.sort at its default (stable=False,
    cvmm.py:1795). At every config size that call returns the stable order on
    B200, and the library's indices equal it bit for bit, so the library
    matches the reference's own CUDA ordering, not just the stable one."""
    from cvmm_codex_b200 import cvmm_prepare_sel2

    g = torch.Generator(device="cuda").manual_seed(R)
    sel = torch.randint(0, E, (R // 4, 4), device="cuda", generator=g)
    fsel = sel.flatten().to(torch.int32)
    default = fsel.sort()
    stable = fsel.sort(stable=True)
    assert torch.equal(default.indices, stable.indices)
    s = cvmm_prepare_sel2(sel)
    assert torch.equal(s.out_index, default.indices)
    assert torch.equal(s.sel.reshape(-1), default.values)
    assert torch.equal(s.sel_index, default.indices // 4)


@pytest.mark.parametrize("src_dtype,dst_dtype,scaled,cols", [
    (torch.bfloat16, torch.bfloat16, False, 136),
    (torch.float32, torch.bfloat16, False, 136),
    (torch.bfloat16, torch.bfloat16, True, 136),
    (torch.float32, torch.float16, True, 136),
    # rows of 1 KiB and more take the warp-per-row kernel (copy and scaled)
    (torch.bfloat16, torch.bfloat16, False, 1032),
    (torch.bfloat16, torch.bfloat16, True, 1024),
    (torch.float16, torch.float16, True, 4104),
])
def test_sort_rows_padded_matches_oracle(src_dtype, dst_dtype, scaled, cols):
    """Expert-padded sorted copy of route rows (the grouping copy of cvmm.py:338-360),
    with the op-dtype rounding and the weighted-grad product rounding of cvmm.py:591-599."""
    g = torch.Generator().manual_seed(21)
    R, E, pad, k = 3000, 11, 128, 3
    sel = torch.randint(0, E, (R // k, k), generator=g)
    sel[:, 0] = 4  # a long segment
    sel[:, 1] = torch.where(sel[:, 1] == 7, 8, sel[:, 1])  # expert 7 empty unless drawn in column 2
    src = torch.randn(R // k, cols, generator=g).to(src_dtype)
    w = torch.rand(R // k, k, generator=g) if scaled else None
    s = C.cvmm_prepare_sel2(sel.cuda(), route_input=True)
    offs = ops.expert_offsets(s.sel, E)
    # NaN-fill a block the caching allocator hands out again, so unwritten padding would show
    junk = torch.full(((R + E * pad) * cols * 4,), float("nan"), device="cuda")
    del junk
    dst, pstart = ops.sort_rows_padded(src.cuda(), s.sel_index, k, s.sel, offs, E, dtype=dst_dtype,
                                       scale=None if w is None else w.cuda())
    _, ssel, idx, _ = O.prepare_sel2(sel.numpy(), route_input=True)
    counts = np.bincount(ssel, minlength=E)
    padded = (counts + pad - 1) // pad * pad
    want_ps = np.concatenate([[0], np.cumsum(padded)[:-1]]).astype(np.int32)
    np.testing.assert_array_equal(pstart.cpu().numpy(), want_ps)
    op = {torch.bfloat16: "bfloat16", torch.float16: "float16"}[dst_dtype]
    want = np.zeros((int(padded.sum()), cols), dtype=np.float64)
    seg = np.concatenate([[0], np.cumsum(counts)[:-1]])
    srcf = src.float().numpy().astype(np.float64)
    for p_ in range(R):
        e = ssel[p_]
        row = O.round_op(srcf[idx[p_] // k], op)
        if w is not None:
            row = O.round_op(row * O.round_op(w.reshape(-1)[idx[p_]].item(), op), op)
        want[want_ps[e] + p_ - seg[e]] = row
    got = dst[: int(padded.sum())].float().cpu().numpy()
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("cols,scaled", [(128, False), (136, True), (1024, False), (1024, True)])
def test_sort_rows_padded_route_rows_matches_map_kernel(cols, scaled):
    """cvmm_sort_rows_padded_ex: the same copy and pad starts as cvmm_sort_rows_padded, and a
    route -> padded row map equal to cvmm_padded_route_rows' (the k-sum's row map), for the
    short-row kernel (128, 136 columns) and the warp-per-row kernel (1024)."""
    g = torch.Generator().manual_seed(5)
    T, k, E = 1500, 4, 13
    sel = torch.randint(0, E, (T, k), generator=g)
    sel[:, 0] = 2  # a segment over several 128-row tiles
    src = torch.randn(T * k, cols, generator=g).to(torch.bfloat16).cuda()
    w = torch.rand(T * k, generator=g).cuda() if scaled else None
    s = C.cvmm_prepare_sel2(sel.cuda())
    offs = ops.expert_offsets(s.sel, E)
    route = s.out_index
    d0, p0 = ops.sort_rows_padded(src, route, 1, s.sel, offs, E, dtype=torch.bfloat16, scale=w)
    d1, p1, rows = ops.sort_rows_padded(src, route, 1, s.sel, offs, E, dtype=torch.bfloat16, scale=w,
                                        route_rows=True)
    used = int(p0[-1].item()) + ((int((offs[-1] - offs[-2]).item()) + 127) // 128) * 128
    assert torch.equal(p0, p1)
    assert torch.equal(d0[:used], d1[:used])
    want = ops.padded_route_rows(route, s.sel, offs, p0)
    assert torch.equal(rows, want)
    # every route's row holds that route's source row
    assert torch.equal(d1[rows.long()], d0[want.long()])
    if w is None:
        assert torch.equal(d1[rows.long()], src)
    # pad starts given, not recomputed: the same copy again
    d2, p2 = ops.sort_rows_padded(src, route, 1, s.sel, offs, E, dtype=torch.bfloat16, scale=w, pad_start=p0)
    assert p2 is p0
    assert torch.equal(d2[:used], d0[:used])


@pytest.mark.parametrize("x_dtype,d_in", [(torch.bfloat16, 256), (torch.float32, 136), (torch.bfloat16, 72)])
def test_forward_x_copy_equals_sorted_copy(x_dtype, d_in):
    """The forward's store-back of the rows it gathers (x_copy) is the
    expert-padded sorted copy that cvmm_sort_rows_padded makes, bit for bit,
    padding rows included; the forward output is unchanged by it."""
    g = torch.Generator().manual_seed(8)
    T, k, E, N = 900, 3, 7, 128
    sel = torch.randint(0, E, (T, k), generator=g)
    sel[: T // 2, 1] = 5  # one expert over several tiles
    x = torch.randn(T, d_in, generator=g).to(x_dtype).cuda()
    keys = (torch.randn(E, d_in, N, generator=g) / d_in ** 0.5).bfloat16().cuda()
    s = C.cvmm_prepare_sel2(sel.cuda())
    offs = ops.expert_offsets(s.sel, E)
    want, wpad = ops.sort_rows_padded(x, s.sel_index, 1, s.sel, offs, E, dtype=torch.bfloat16)
    pad = ops.pad_starts(offs, E)
    assert torch.equal(pad, wpad)
    xs = torch.full_like(want, float("nan"))
    y = ops.forward(x, s.sel_index, offs, keys, s.out_index, torch.bfloat16, torch.bfloat16, x_copy=xs)
    used = int(pad[-1].item()) + (int(offs[-1].item() - (offs[-2].item() if E > 1 else 0)) + 127) // 128 * 128
    assert torch.equal(xs[:used], want[:used])
    y_ref = ops.forward(x, s.sel_index, offs, keys, s.out_index, torch.bfloat16, torch.bfloat16)
    assert torch.equal(y, y_ref)
