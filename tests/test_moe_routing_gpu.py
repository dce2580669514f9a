"""Device MoE routing (router softmax / top-k kernel, expert-major layout and
copy rows built on the GPU) against torch and the host-built layouts."""

import pytest
import torch

pytestmark = pytest.mark.gpu

PAD = 128


@pytest.mark.parametrize("E,k,norm,bf16", [(128, 8, True, False), (64, 4, False, True), (8, 2, True, False)])
def test_moe_route_matches_torch(cuda_ext, E, k, norm, bf16):
    torch.manual_seed(E + k)
    T = 777
    logits = torch.randn(T, E, device="cuda") * 2
    probs = torch.empty(T, E, device="cuda")
    topi = torch.empty(T, k, device="cuda", dtype=torch.int64)
    topv = torch.empty(T, k, device="cuda")
    w = torch.empty(T, k, device="cuda")
    s = torch.empty(T, 1, device="cuda")
    counts = torch.zeros(E, device="cuda", dtype=torch.int32)
    cuda_ext.moe_route(logits, k, norm, bf16, probs, topi, topv, w, s, counts)
    lg = logits.to(torch.bfloat16).float() if bf16 else logits
    p_ref = torch.softmax(lg, -1)
    torch.testing.assert_close(probs, p_ref, rtol=1e-5, atol=1e-6)
    v_ref, i_ref = torch.topk(p_ref, k, -1)
    torch.testing.assert_close(topv, v_ref, rtol=1e-5, atol=1e-6)
    # same expert sets (order within exact ties may differ)
    assert torch.equal(torch.sort(topi, -1).values, torch.sort(i_ref, -1).values) or \
        (p_ref.gather(1, topi) - v_ref).abs().max() < 1e-6
    torch.testing.assert_close(s[:, 0], topv.sum(-1), rtol=1e-5, atol=1e-6)
    want_w = topv / topv.sum(-1, keepdim=True) if norm else topv
    torch.testing.assert_close(w, want_w, rtol=1e-5, atol=1e-6)
    assert torch.equal(counts.long(), torch.bincount(topi.flatten(), minlength=E))


def _layout(cuda_ext, allc, ep, me, E, cap):
    El = E // ep
    dev = allc.device
    base = torch.empty(E, dtype=torch.int64, device=dev)
    tg = torch.empty(cap // PAD, dtype=torch.int32, device=dev)
    ks, kl, nr = (torch.empty(El, dtype=torch.int32, device=dev) for _ in range(3))
    rows = torch.empty(1, dtype=torch.int32, device=dev)
    ov = torch.empty(1, dtype=torch.int32, device=dev)
    cuda_ext.moe_layout(allc, ep, me, PAD, cap, base, tg, ks, kl, nr, rows, ov)
    return base, tg, ks, kl, nr, int(rows), int(ov)


def test_local_layout_matches_host_routing(cuda_ext):
    from wavelet_b200.models.moe import Routing

    torch.manual_seed(3)
    T, k, E = 500, 8, 64
    topi = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)])
    topi[:40] = torch.arange(k, device="cuda")  # a crowded expert block
    counts = torch.bincount(topi.flatten(), minlength=E).to(torch.int32)
    host = Routing(topi, E)
    cap = (T * k + E * (PAD - 1) + PAD - 1) // PAD * PAD
    base, tg, ks, kl, nr, rows, ov = _layout(cuda_ext, counts, 1, 0, E, cap)
    assert ov == 0 and rows == host.R
    assert torch.equal(ks, host.k_start) and torch.equal(kl, host.k_len)
    assert torch.equal(nr.long(), counts.long())
    ntiles = host.R // PAD
    assert torch.equal(tg[:ntiles], host.tile_group[:ntiles]) and bool((tg[ntiles:] == -1).all())
    pos = torch.empty(T * k, dtype=torch.int64, device="cuda")
    rank = torch.empty(T * k, dtype=torch.int32, device="cuda")
    cuda_ext.moe_copy_rows(topi.flatten().contiguous(), E, E, base, pos, rank)
    assert torch.equal(pos, host.pos) and bool((rank == 0).all())


def test_ep_layout_matches_host_formula_and_reports_overflow(cuda_ext):
    torch.manual_seed(5)
    ep, E, k, T = 4, 32, 4, 300
    El = E // ep
    C = torch.randint(0, 60, (ep, E), device="cuda", dtype=torch.int32)
    Ch = C.tolist()
    for me in range(ep):
        cap = 64 * PAD
        base, tg, ks, kl, nr, rows, ov = _layout(cuda_ext, C.flatten().contiguous(), ep, me, E, cap)
        assert ov == 0
        seg = {}
        for d in range(ep):
            acc = 0
            for el in range(El):
                seg[(d, el)] = acc
                n = sum(Ch[s][d * El + el] for s in range(ep))
                acc += (n + PAD - 1) // PAD * PAD
        for ge in range(E):
            d, el = divmod(ge, El)
            assert int(base[ge]) == seg[(d, el)] + sum(Ch[s][ge] for s in range(me))
        for el in range(El):
            n = sum(Ch[s][me * El + el] for s in range(ep))
            assert int(ks[el]) == seg[(me, el)] and int(kl[el]) == (n + PAD - 1) // PAD * PAD and int(nr[el]) == n
    # a capacity no layout fits: flag + error bit, empty tile map
    cuda_ext.clear_error(0)
    base, tg, ks, kl, nr, rows, ov = _layout(cuda_ext, C.flatten().contiguous(), ep, 0, E, 2 * PAD)
    assert ov == 1 and bool((tg == -1).all())
    assert cuda_ext.read_error(0) & (1 << 6)
    cuda_ext.clear_error(0)


def test_rows_exchange_skips_rows_past_the_limit(cuda_ext):
    from wavelet_b200.parallel.fabric import Fabric

    fab = Fabric(0, 1, torch.device("cuda", 0))
    H, R = 128, 64
    buf = fab.alloc((R + 8) * H, torch.bfloat16)  # 8 sentinel rows past the limit
    buf.tensor.fill_(7.0)
    x = torch.randn(10, H, device="cuda", dtype=torch.bfloat16)
    src = torch.arange(10, device="cuda")
    rank = torch.zeros(10, device="cuda", dtype=torch.int32)
    row = torch.tensor([0, 1, 2, 63, 64, 65, 70, -1, 5, 6], device="cuda")
    cuda_ext.rows_scatter(x, src, rank, row, None, [buf.ptrs[0]], 1, H, R)
    v = buf.tensor.view(R + 8, H)
    assert bool((v[R:] == 7.0).all())  # nothing written past the limit
    assert torch.equal(v[63], x[3]) and torch.equal(v[0], x[0])
    out = torch.empty(10, H, device="cuda", dtype=torch.float32)
    cuda_ext.rows_gather_sum([buf.ptrs[0]], 1, H, rank, row, None, 1, None, out, R)
    assert bool((out[4:8] == 0).all())  # rows past the limit read as nothing
    torch.testing.assert_close(out[3], x[3].float())
    fab.close()
