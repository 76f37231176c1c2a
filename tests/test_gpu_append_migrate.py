"""KV append and KV migration on the device, bit-exact against the oracle."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import make_tables

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _append_case(seed, T, Hkv, D, BS, nseq=3):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 5 * BS, nseq).astype(np.int32)
    nb = int(sum((c + BS - 1) // BS for c in ctx)) + 2
    bt = make_tables(ctx, BS, nb, rng)
    tok_seq = rng.integers(0, nseq, T).astype(np.int32)
    tok_pos = np.array([rng.integers(0, ctx[s]) for s in tok_seq], np.int32)
    # distinct (seq, pos) so that rows never overwrite each other
    _, keep = np.unique(tok_seq * 100000 + tok_pos, return_index=True)
    tok_seq, tok_pos = tok_seq[np.sort(keep)], tok_pos[np.sort(keep)]
    T = len(tok_seq)
    key = rng.standard_normal((T, Hkv, D)).astype(np.float32) * 3
    val = rng.standard_normal((T, Hkv, D)).astype(np.float32) * 3
    key[0, 0] = 0.0                        # all-zero row -> scale 1.0
    key[-1, -1, :4] = [2.5, -2.5, 0.5, -0.5]
    return nb, bt, tok_seq, tok_pos, key, val


@pytest.mark.parametrize("storage", ["fp32", "int8", "int4"])
def test_append_bit_exact(cuda_device, storage):
    from gollek_b200 import ops
    Hkv, D, BS = 4, 64, 16
    nb, bt, ts, tp, key, val = _append_case(3, 40, Hkv, D, BS)
    st = O.STORAGE[storage]
    bbytes = O.block_bytes(st, Hkv, BS, D)
    if st == O.FP32:
        ks_ = kv_ = None
        k_slab = np.zeros((nb, Hkv, BS, D), np.float32)
    else:
        k_slab = np.zeros(nb * bbytes, np.uint8)
    v_slab = np.zeros_like(k_slab)
    k_sc = np.zeros(nb * Hkv * BS, np.float32) if st != O.FP32 else None
    v_sc = np.zeros_like(k_sc) if st != O.FP32 else None
    rc = O.update_cache(key, val, tp, bt, storage=st, k_slab=k_slab, v_slab=v_slab,
                        k_scale=k_sc, v_scale=v_sc, token_seq=ts, block_size=BS)
    assert rc == 0
    dk = torch.zeros(k_slab.shape, dtype=torch.float32 if st == O.FP32 else torch.uint8,
                     device=cuda_device)
    dv = torch.zeros_like(dk)
    dks = torch.zeros(nb * Hkv * BS, device=cuda_device) if st != O.FP32 else None
    dvs = torch.zeros_like(dks) if st != O.FP32 else None
    if st == O.INT8:
        dk, dv = dk.view(torch.int8), dv.view(torch.int8)
    ops.kv_append(_t(key, cuda_device), _t(val, cuda_device), _t(tp, cuda_device),
                  _t(bt, cuda_device), dk, dv, block_size=BS, num_blocks=nb,
                  token_seq=_t(ts, cuda_device), k_scales=dks, v_scales=dvs,
                  scale_strides=(Hkv * BS, BS, 1), int4=(st == O.INT4))
    torch.cuda.synchronize()
    got_k = dk.cpu().numpy().view(k_slab.dtype).reshape(k_slab.shape)
    got_v = dv.cpu().numpy().view(v_slab.dtype).reshape(v_slab.shape)
    assert np.array_equal(got_k.view(np.uint8), k_slab.view(np.uint8))
    assert np.array_equal(got_v.view(np.uint8), v_slab.view(np.uint8))
    if st != O.FP32:
        assert np.array_equal(dks.cpu().numpy().view(np.uint32), k_sc.view(np.uint32))
        assert np.array_equal(dvs.cpu().numpy().view(np.uint32), v_sc.view(np.uint32))


def test_append_bf16_pool_from_fp32(cuda_device):
    from gollek_b200 import ops
    Hkv, D, BS = 8, 128, 16
    nb, bt, ts, tp, key, val = _append_case(4, 64, Hkv, D, BS)
    dk = torch.zeros((nb, Hkv, BS, D), dtype=torch.bfloat16, device=cuda_device)
    dv = torch.zeros_like(dk)
    ops.kv_append(_t(key, cuda_device), _t(val, cuda_device), _t(tp, cuda_device),
                  _t(bt, cuda_device), dk, dv, block_size=BS, num_blocks=nb,
                  token_seq=_t(ts, cuda_device))
    ref_k = np.zeros((nb, Hkv, BS, D), np.float32)
    ref_v = np.zeros_like(ref_k)
    O.update_cache(key, val, tp, bt, storage=O.FP32, k_slab=ref_k, v_slab=ref_v, token_seq=ts,
                   block_size=BS)
    assert np.array_equal(dk.float().cpu().numpy(), O.round_bf16(ref_k))
    assert np.array_equal(dv.float().cpu().numpy(), O.round_bf16(ref_v))


def test_append_then_decode_matches_oracle(cuda_device):
    """The engine's order: updateCache for the new token, then attention over ctx+1."""
    from gollek_b200 import ops
    from tests.helpers import decode_case, oracle_decode
    ctx = [15, 16, 100, 257]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=9, spare_pages=8,
                                   max_blocks=20)
    # give every sequence room for one more token
    for s, c in enumerate(ctx):
        if c % 16 == 0:
            used = set(bt[bt >= 0].tolist())
            free = [p for p in range(k.shape[0]) if p not in used]
            bt[s, c // 16] = free[0]
    rng = np.random.default_rng(10)
    newk = rng.standard_normal((4, 8, 128)).astype(np.float32)
    newv = rng.standard_normal((4, 8, 128)).astype(np.float32)
    pos = ctx.copy()
    kd, vd = _t(k, cuda_device), _t(v, cuda_device)
    ops.kv_append(_t(newk, cuda_device), _t(newv, cuda_device), _t(pos, cuda_device),
                  _t(bt, cuda_device), kd, vd, block_size=16, num_blocks=k.shape[0])
    O.update_cache(newk, newv, pos, bt, storage=O.FP32, k_slab=k, v_slab=v, block_size=16)
    ctx1 = ctx + 1
    want = oracle_decode(q, k, v, bt, ctx1, 1 / np.sqrt(128), hkv=8, bs=16)
    out = ops.paged_attention(_t(q, cuda_device), kd, vd, _t(bt, cuda_device),
                              _t(ctx1, cuda_device), num_kv_heads=8, block_size=16,
                              num_blocks=k.shape[0])
    err = np.abs(out.cpu().numpy() - want).max()
    assert err <= 1e-4 * np.abs(want).max()


def test_migrate_same_device_bit_exact(cuda_device):
    """transferKvToDecodePartition within one pool: [block][layer][bytes] slices."""
    from gollek_b200 import ops
    L, H, BS, D = 4, 2, 16, 32
    bpb = BS * H * D * 2  # bf16 bytes per (block, layer)
    nb = 24
    rng = np.random.default_rng(12)
    k = rng.integers(0, 256, nb * L * bpb, dtype=np.uint8)
    v = rng.integers(0, 256, nb * L * bpb, dtype=np.uint8)
    src = np.array([0, 3, 5, 7, 2], np.int32)
    dst = np.array([20, 13, 17, 12, 23], np.int32)
    kk, vv = k.copy(), v.copy()
    O.migrate(kk, vv, kk, vv, src, dst, L, bpb)
    dk, dv = _t(k, cuda_device), _t(v, cuda_device)
    ops.kv_migrate(dk, dv, dk, dv, _t(src, cuda_device), _t(dst, cuda_device),
                   src_block_stride=L * bpb, dst_block_stride=L * bpb, bytes_per_block=L * bpb)
    torch.cuda.synchronize()
    assert np.array_equal(dk.cpu().numpy(), kk) and np.array_equal(dv.cpu().numpy(), vv)


def test_migrate_unaligned_bytes_path(cuda_device):
    from gollek_b200 import ops
    rng = np.random.default_rng(13)
    a = rng.integers(0, 256, 9 * 37, dtype=np.uint8)
    b = np.zeros(9 * 37, np.uint8)
    src = np.array([1, 8, 4], np.int32)
    dst = np.array([0, 2, 7], np.int32)
    ref = b.copy()
    for s, d in zip(src, dst):
        ref[d * 37:(d + 1) * 37] = a[s * 37:(s + 1) * 37]
    da, db = _t(a, cuda_device), _t(b, cuda_device)
    ops.kv_migrate(da, None, db, None, _t(src, cuda_device), _t(dst, cuda_device),
                   src_block_stride=37, dst_block_stride=37, bytes_per_block=37)
    torch.cuda.synchronize()
    assert np.array_equal(db.cpu().numpy(), ref)


def test_migrate_skips_out_of_range_ids(cuda_device):
    """Ids outside a pool (negative, or >= the pool's block count) are skipped on the
    device and raise GOLLEK_STATUS_BAD_BLOCK_ID; the valid copies of the same call land.
    The ids are checked before any address is formed, so nothing outside the pools is
    touched (local memory only)."""
    from gollek_b200 import _lib, ops
    ops.device_status(cuda_device.index, clear=True)
    bpb, nb = 4096, 12
    rng = np.random.default_rng(21)
    a = rng.integers(0, 256, nb * bpb, dtype=np.uint8)
    b = rng.integers(0, 256, nb * bpb, dtype=np.uint8)
    src = np.array([1, nb, 4, -1, 6], np.int32)
    dst = np.array([0, 2, nb + 5, 9, 11], np.int32)
    ref = b.copy()
    for s_, d_ in zip(src, dst):
        if 0 <= s_ < nb and 0 <= d_ < nb:
            ref[d_ * bpb:(d_ + 1) * bpb] = a[s_ * bpb:(s_ + 1) * bpb]
    da, db = _t(a, cuda_device), _t(b, cuda_device)
    ops.kv_migrate(da, None, db, None, _t(src, cuda_device), _t(dst, cuda_device),
                   src_block_stride=bpb, dst_block_stride=bpb, bytes_per_block=bpb)
    torch.cuda.synchronize()
    assert np.array_equal(db.cpu().numpy(), ref)
    assert ops.device_status(cuda_device.index, clear=True) & _lib.STATUS_BAD_BLOCK_ID
    # the byte-granular kernel checks the same way
    db2 = _t(b, cuda_device)
    ops.kv_migrate(da[:nb * bpb - 3], None, db2, None, _t(src, cuda_device), _t(dst, cuda_device),
                   src_block_stride=bpb, dst_block_stride=bpb, bytes_per_block=bpb - 3)
    torch.cuda.synchronize()
    ref2 = b.copy()
    for s_, d_ in zip(src, dst):
        if 0 <= s_ < nb and 0 <= d_ < nb:
            ref2[d_ * bpb:d_ * bpb + bpb - 3] = a[s_ * bpb:s_ * bpb + bpb - 3]
    assert np.array_equal(db2.cpu().numpy(), ref2)
    assert ops.device_status(cuda_device.index, clear=True) & _lib.STATUS_BAD_BLOCK_ID
    # checksums: a bad id reads nothing and reports 0
    got = ops.block_checksums(da, _t(np.array([3, nb, -2], np.int32), cuda_device),
                              block_stride=bpb, bytes_per_block=bpb).cpu().numpy()
    assert got[1] == 0 and got[2] == 0 and got[0] != 0
    assert ops.device_status(cuda_device.index, clear=True) & _lib.STATUS_BAD_BLOCK_ID
    # a clean call leaves the status clear
    ops.kv_migrate(da, None, db, None, _t(np.array([2], np.int32), cuda_device),
                   _t(np.array([3], np.int32), cuda_device), src_block_stride=bpb,
                   dst_block_stride=bpb, bytes_per_block=bpb)
    assert ops.device_status(cuda_device.index, clear=True) == 0


def test_block_checksums_match_numpy(cuda_device):
    from gollek_b200 import ops
    rng = np.random.default_rng(14)
    nb, bpb = 10, 4096
    pool = rng.integers(0, 256, nb * bpb, dtype=np.uint8)
    blocks = np.array([9, 0, 4], np.int32)
    got = ops.block_checksums(_t(pool, cuda_device), _t(blocks, cuda_device), block_stride=bpb,
                              bytes_per_block=bpb).cpu().numpy().view(np.uint64)
    w = pool.view(np.uint64).reshape(nb, -1)
    j = np.arange(w.shape[1], dtype=np.uint64)
    mix = j * np.uint64(0x9E3779B97F4A7C15)
    want = [(w[b] ^ mix).sum(dtype=np.uint64) for b in blocks]
    assert list(got) == want


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_migrate_peer_bit_exact():
    """Source pool on GPU 0, destination on GPU 1, remapped: bytes equal, checksums equal."""
    from gollek_b200 import ops
    ops.enable_peer_access(0, 1)
    L, bpb, nb = 8, 32 * 1024, 40
    d0, d1 = torch.device("cuda:0"), torch.device("cuda:1")
    g = torch.Generator(device=d0).manual_seed(3)
    sk = torch.randint(0, 256, (nb * L * bpb,), dtype=torch.uint8, device=d0, generator=g)
    sv = torch.randint(0, 256, (nb * L * bpb,), dtype=torch.uint8, device=d0, generator=g)
    dk = torch.zeros(nb * L * bpb, dtype=torch.uint8, device=d1)
    dv = torch.zeros_like(dk)
    rng = np.random.default_rng(4)
    src = rng.permutation(nb)[:25].astype(np.int32)
    dst = rng.permutation(nb)[:25].astype(np.int32)
    ops.kv_migrate(sk, sv, dk, dv, _t(src, d0), _t(dst, d0), src_block_stride=L * bpb,
                   dst_block_stride=L * bpb, bytes_per_block=L * bpb, device=0)
    torch.cuda.synchronize(d0)
    skn, dkn = sk.cpu().numpy().reshape(nb, -1), dk.cpu().numpy().reshape(nb, -1)
    svn, dvn = sv.cpu().numpy().reshape(nb, -1), dv.cpu().numpy().reshape(nb, -1)
    for s, d in zip(src, dst):
        assert np.array_equal(skn[s], dkn[d]) and np.array_equal(svn[s], dvn[d])
