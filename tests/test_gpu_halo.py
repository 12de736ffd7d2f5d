"""The K/V halo of the spatial partition on one GPU: the ring-write kernel's
stores of a strip's edge columns into the neighbours' rings, its signal, and the
bounded counter wait. The neighbours' rings here are buffers of the same GPU,
so the addressing and the counters are checked without a second GPU (the
2-GPU model tests run the same kernels over NVLink)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ring_write_stores_the_halo_columns_and_signals(srdit, cuda_device):
    L = srdit._lib
    dev = cuda_device
    f, h, wl, R, D, cap, slot0 = 3, 4, 8, 3, 256, 5, 3   # slots 3, 4, 0: the ring wraps
    We = wl + 2 * R            # a middle strip: halo on both sides, own columns at [R, R + wl)
    Wl, Wr = wl + 2 * R, wl + R  # the left neighbour a middle strip, the right one the last
    M = f * h * wl
    g = torch.Generator().manual_seed(11)
    src = torch.randn(M, D, generator=g).to(torch.bfloat16).to(dev)
    vsrc = torch.randn(M, D, generator=g).to(torch.bfloat16).to(dev)
    weight = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(dev)

    def zeros(width):
        return torch.zeros(cap * h * width, D, dtype=torch.bfloat16, device=dev)

    common = dict(frame_tokens=h * wl, slot0=slot0, n_slots=cap, grid_h=h, grid_w=wl,
                  dst_grid_w=We, dst_w0=R)
    ref_k, ref_v = zeros(We), zeros(We)
    srdit.ops.rms_rope(src, weight, 1e-6, ref_k, v_src=vsrc, v_dst=ref_v, **common)

    ring_k, ring_v = zeros(We), zeros(We)
    left_k, left_v, right_k, right_v = zeros(Wl), zeros(Wl), zeros(Wr), zeros(Wr)
    flags = torch.zeros(8, dtype=torch.int32, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    hs = L.RopeHalo()
    # left: this strip's columns [0, R) at the left neighbour's columns [R + wl, Wl)
    hs.k[0], hs.v[0], hs.grid_w[0], hs.w0[0] = left_k.data_ptr(), left_v.data_ptr(), Wl, R + wl
    hs.col_lo[0], hs.col_hi[0], hs.flag[0] = 0, R, flags.data_ptr() + 4 * 2
    # right: columns [wl - R, wl) at the right neighbour's columns [0, R)
    hs.k[1], hs.v[1], hs.grid_w[1], hs.w0[1] = right_k.data_ptr(), right_v.data_ptr(), Wr, R - wl
    hs.col_lo[1], hs.col_hi[1], hs.flag[1] = wl - R, wl, flags.data_ptr() + 4 * 5
    hs.done = done.data_ptr()
    for _ in range(2):
        srdit.ops.rms_rope(src, weight, 1e-6, ring_k, v_src=vsrc, v_dst=ring_v, halo=hs, **common)
    torch.cuda.synchronize(dev)

    assert torch.equal(ring_k, ref_k) and torch.equal(ring_v, ref_v)
    slots = [(slot0 + j) % cap for j in range(f)]
    for ref, left, right in ((ref_k, left_k, right_k), (ref_v, left_v, right_v)):
        r4 = ref.view(cap, h, We, D)
        l4, q4 = left.view(cap, h, Wl, D), right.view(cap, h, Wr, D)
        exp_l, exp_r = torch.zeros_like(l4), torch.zeros_like(q4)
        for s in slots:
            exp_l[s, :, R + wl:] = r4[s, :, R:2 * R]
            exp_r[s, :, :R] = r4[s, :, wl:wl + R]
        assert torch.equal(l4, exp_l) and torch.equal(q4, exp_r)
    # one signal per launch in each neighbour's counter of this rank; `done` back at 0
    assert flags.tolist() == [0, 0, 2, 0, 0, 2, 0, 0]
    assert int(done.item()) == 0


def test_ring_write_rejects_halo_columns_outside_the_neighbour(srdit, cuda_device):
    L = srdit._lib
    dev = cuda_device
    h, wl, D = 2, 8, 128
    src = torch.zeros(h * wl, D, dtype=torch.bfloat16, device=dev)
    weight = torch.ones(D, dtype=torch.bfloat16, device=dev)
    ring = torch.zeros(2 * h * wl, D, dtype=torch.bfloat16, device=dev)
    peer = torch.zeros_like(ring)
    flags = torch.zeros(8, dtype=torch.int32, device=dev)
    hs = L.RopeHalo()
    hs.k[0], hs.grid_w[0], hs.w0[0], hs.col_lo[0], hs.col_hi[0] = peer.data_ptr(), wl, 1, 0, wl
    hs.flag[0], hs.done = flags.data_ptr(), flags.data_ptr() + 4
    with pytest.raises(L.SrditError):   # columns 1..8 of an 8-column frame
        srdit.ops.rms_rope(src, weight, 1e-6, ring, frame_tokens=h * wl, n_slots=2, grid_h=h,
                           grid_w=wl, dst_grid_w=wl, dst_w0=0, halo=hs)
    assert int(flags.sum().item()) == 0


def test_counter_wait_returns_and_times_out(srdit, cuda_device):
    """The wait returns at once when the counters are reached and, when one never
    is (nothing signals it), gives up after its time budget with the timeout
    status instead of hanging."""
    dev = cuda_device
    counters = torch.tensor([1, 0, 1, 0, 0, 0, 0, 0], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    srdit.ops.wait_counters(counters.data_ptr(), 0b101, 1, status=status, device=dev)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0
    srdit.ops.wait_counters(counters.data_ptr(), 0b111, 1, status=status, device=dev)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == srdit._lib.SRDIT_STATUS_TIMEOUT
