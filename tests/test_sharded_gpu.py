"""GPU tests of the sharded step: every sharding / bucketing of the same parameter set must produce
the same bits as the unsharded one (groups never straddle a cut), checked on one GPU by running the
ranks' local steps one after the other (no collective; the gather itself is covered by the gloo
tests of the plan and by the multi-GPU bench)."""
import pytest
import torch

from coat_b200.sharded import GROUP, ShardedCoatAdamW

pytestmark = pytest.mark.gpu

HYPER = dict(lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, expand_min=16)
NUMELS = [128 * 37, 77, 128 * 3 + 1, 4096 * 8, 1, 128 * 128, 300]


def fill(opt, seed):
    """Every element's value depends only on (tensor, element index), not on who owns it."""
    for pc in opt.my_pieces:
        gen = torch.Generator().manual_seed(seed * 1000 + pc.tensor)
        n = NUMELS[pc.tensor]
        p = torch.randn(n, generator=gen) * 0.02
        g = torch.randn(n, generator=gen) * 1e-3
        opt.param[pc.offset:pc.offset + pc.numel] = p[pc.start:pc.stop].cuda()
        opt.grad[pc.offset:pc.offset + pc.numel] = g[pc.start:pc.stop].cuda()


def collect(opts):
    """Per tensor: fp32 weights, codes, per-group vectors, bf16 copy, assembled from all ranks' pieces."""
    out = {}
    for opt in opts:
        for pc in opt.my_pieces:
            o, go, ng = pc.offset, pc.offset // GROUP, (pc.numel + GROUP - 1) // GROUP
            bo = opt.plan.gathered_offset(opt.rank, o, opt.n_buckets)
            rec = dict(p=opt.param[o:o + pc.numel], m=opt.exp_avg[o:o + pc.numel], v=opt.exp_avg_sq[o:o + pc.numel],
                       s_m=opt.scale_exp_avg[go:go + ng], k_m=opt.expand_exp_avg[go:go + ng],
                       r_m=opt.sqrt_minmax_exp_avg[go:go + ng], s_v=opt.scale_exp_avg_sq[go:go + ng],
                       k_v=opt.expand_exp_avg_sq[go:go + ng], r_v=opt.sqrt_minmax_exp_avg_sq[go:go + ng],
                       bf16=opt.gathered[bo:bo + pc.numel])
            out.setdefault(pc.tensor, []).append((pc.start, {k: v.clone().cpu() for k, v in rec.items()}))
    merged = {}
    for t, lst in out.items():
        lst.sort(key=lambda x: x[0])
        merged[t] = {k: torch.cat([r[k] for _, r in lst]) for k in lst[0][1]}
    return merged


def run(world, buckets, steps=3):
    # ranks are emulated one after the other on one GPU: only local_step() runs, no exchange is set up
    opts = [ShardedCoatAdamW(NUMELS, rank=r, world_size=world, device="cuda", n_buckets=buckets,
                             exchange="nccl" if world > 1 else None, **HYPER)
            for r in range(world)]
    for s in range(steps):
        for opt in opts:
            fill_grad_only = s > 0
            if not fill_grad_only:
                fill(opt, 0)
            else:   # new gradients every step, same weights carried over
                for pc in opt.my_pieces:
                    gen = torch.Generator().manual_seed(s * 1000 + pc.tensor)
                    g = torch.randn(NUMELS[pc.tensor], generator=gen) * 1e-3
                    opt.grad[pc.offset:pc.offset + pc.numel] = g[pc.start:pc.stop].cuda()
            opt.local_step()
    torch.cuda.synchronize()
    return collect(opts)


@pytest.mark.parametrize("world,buckets", [(1, 3), (2, 1), (2, 5), (3, 8)])
def test_sharded_and_bucketed_steps_equal_the_unsharded_step(world, buckets):
    want = run(1, 1)
    got = run(world, buckets)
    assert want.keys() == got.keys()
    for t in want:
        for k in want[t]:
            a, b = want[t][k], got[t][k]
            assert a.shape == b.shape, (t, k)
            assert torch.equal(a.view(torch.uint8) if a.dtype != torch.uint8 else a,
                               b.view(torch.uint8) if b.dtype != torch.uint8 else b), (t, k)


def test_weight_views_cover_every_tensor():
    opt = ShardedCoatAdamW(NUMELS, rank=0, world_size=1, device="cuda", n_buckets=4, **HYPER)
    fill(opt, 0)
    opt.local_step()
    torch.cuda.synchronize()
    views = opt.weight_views([(n,) for n in NUMELS])
    got = collect([opt])
    for t, v in enumerate(views):
        flat = v if isinstance(v, torch.Tensor) else torch.cat(v)
        assert flat.numel() == NUMELS[t]
        assert torch.equal(flat.cpu().view(torch.int16), got[t]["bf16"].view(torch.int16))


def test_set_grad_buffer_rejects_wrong_size():
    opt = ShardedCoatAdamW(NUMELS, rank=0, world_size=1, device="cuda", **HYPER)
    with pytest.raises(ValueError):
        opt.set_grad_buffer(torch.zeros(5, device="cuda"))


def test_broadcast_step_writes_every_peer_copy():
    """The broadcast kernel with two stand-in peers (plain buffers on the same GPU): both receive the
    bf16 slice at the same offsets, and weights / state are those of the plain table launch."""
    import ctypes
    want = run(1, 1, steps=2)
    opt = ShardedCoatAdamW(NUMELS, rank=0, world_size=1, device="cuda", **HYPER)
    peers = [torch.full_like(opt.gathered, 7.0) for _ in range(2)]
    opt._peer_deltas = (ctypes.c_int64 * 2)(*[p.data_ptr() - opt.gathered.data_ptr() for p in peers])
    for s in range(2):
        if s == 0:
            fill(opt, 0)
        else:
            for pc in opt.my_pieces:
                gen = torch.Generator().manual_seed(s * 1000 + pc.tensor)
                g = torch.randn(NUMELS[pc.tensor], generator=gen) * 1e-3
                opt.grad[pc.offset:pc.offset + pc.numel] = g[pc.start:pc.stop].cuda()
        opt.step_count += 1
        opt._launch_bucket(0, bcast=True)
    torch.cuda.synchronize()
    got = collect([opt])
    for t in want:
        for k in want[t]:
            assert torch.equal(want[t][k].view(torch.uint8), got[t][k].view(torch.uint8)), (t, k)
    for pc in opt.my_pieces:   # padding between pieces stays untouched in the peers (still 7.0)
        o = opt.plan.gathered_offset(0, pc.offset, 1)
        for p in peers:
            assert torch.equal(p[o:o + pc.numel].view(torch.int16), opt.gathered[o:o + pc.numel].view(torch.int16))
    touched = sum(pc.numel for pc in opt.my_pieces)
    for p in peers:
        assert int((p != 7.0).sum()) <= touched


def test_broadcast_step_argument_checks():
    import ctypes
    from coat_b200 import _lib
    opt = ShardedCoatAdamW(NUMELS, rank=0, world_size=1, device="cuda", **HYPER)
    table, prefix, n_pieces, n_groups = opt._tables[0]
    L = _lib.lib()

    def call(deltas, n):
        arr = (ctypes.c_int64 * max(len(deltas), 1))(*deltas) if deltas is not None else None
        return L.coat_fp8_adamw_multi_step_bcast(table.data_ptr(), prefix.data_ptr(), n_pieces, n_groups, 1, 0.9, 0.95,
                                                 1e-4, 0.1, 1e-8, 1, GROUP, 16, _lib.F32, 0, arr, n,
                                                 _lib.stream_ptr(opt.device))
    assert call([0] * 8, 8) == -1          # more than COAT_MAX_PEERS
    assert call(None, 1) == -1             # peers announced, no deltas
    assert call([8], 1) == -3              # a delta that breaks the 16-byte alignment of the bulk stores
    torch.cuda.synchronize()


def test_peer_buffer_round_trip_in_one_process():
    from coat_b200 import _lib
    from coat_b200.sharded import _PeerBuffer
    buf = _PeerBuffer(_lib, 1 << 20, torch.device("cuda", 0))
    assert len(buf.handle) == _lib.PEER_HANDLE_BYTES and buf.ptr % 256 == 0
    t = torch.as_tensor(buf, device="cuda").view(torch.bfloat16)
    assert t.data_ptr() == buf.ptr and t.numel() == (1 << 19) and not t.any()
    t.fill_(3.0)
    assert float(t.float().sum()) == 3.0 * (1 << 19)
    del t
    torch.cuda.synchronize()
    buf.free()
