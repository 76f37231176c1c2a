"""Pins the CPU oracle to the known answers in the reference's own unit tests.

Each test restates one reference test case (cited by file:line) against the C
restatement in oracle/oracle.c.  Reference paths are relative to its project root:
  PAT/ = optimization/gollek-plugin-paged-attention/src/test/java/tech/kayys/gollek/kernel/paged/
  STT/ = runner/safetensor/gollek-safetensor-engine/src/test/java/tech/kayys/gollek/safetensor/engine/
"""
import math

import numpy as np
import pytest

from oracle import oracle as O


# ------------------------------------------- PagedAttentionCpuFallbackTest

def test_fallback_single_sequence_single_head():
    """PAT/PagedAttentionCpuFallbackTest.java:35-97."""
    q = np.array([[[1.0, 0.0]]], np.float32)
    k = np.zeros((1, 1, 4, 2), np.float32)
    v = np.zeros((1, 1, 4, 2), np.float32)
    k[0, 0, 0] = [1.0, 0.0]
    k[0, 0, 1] = [0.0, 1.0]
    v[0, 0, 0] = [1.0, 0.0]
    v[0, 0, 1] = [0.0, 1.0]
    bt = np.array([[0]], np.int32)
    ctx = np.array([2], np.int32)
    scale = np.float32(1.0) / np.float32(math.sqrt(2))
    out = O.a1_execute(q, k, v, bt, ctx, scale)
    out0, out1 = out[0, 0]
    assert out0 > 0.5
    assert out1 < 0.5
    assert abs((out0 + out1) - 1.0) <= 0.001
    # The test's own comment: softmax([0.707, 0]) ~= [0.669, 0.331].
    assert abs(out0 - 0.6697) < 1e-3


def test_fallback_multiple_blocks_mean_of_v():
    """PAT/PagedAttentionCpuFallbackTest.java:99-148: uniform scores -> mean(V) = 4.0."""
    q = np.array([[[1.0]]], np.float32)
    k = np.array([1.0, 1.0, 1.0, 0.0], np.float32).reshape(2, 1, 2, 1)
    v = np.array([2.0, 4.0, 6.0, 0.0], np.float32).reshape(2, 1, 2, 1)
    bt = np.array([[0, 1]], np.int32)
    ctx = np.array([3], np.int32)
    out = O.a1_execute(q, k, v, bt, ctx, 1.0)
    assert abs(out[0, 0, 0] - 4.0) <= 0.001


# ------------------------------------------------ PagedAttentionVectorMath

def test_vector_math_fp32():
    """STT/generation/attention/PagedAttentionVectorMathTest.java:20-39."""
    q = np.array([1, 2, 3, 4], np.float32)
    key = np.array([0.5, -1, 2, 1], np.float32)
    value = np.array([10, 20, 30, 40], np.float32)
    acc = np.array([1, 2, 3, 4], np.float32)
    for lanes in (1, 2, 4, 8, 16):
        s = O.score(O.FP32, q, key, dim=4, scale=0.5, lanes=lanes)
        assert abs(s - 4.25) <= 1e-4
    acc = O.update(O.FP32, acc, value, prev=0.5, cur=0.25)
    np.testing.assert_allclose(acc, [3, 6, 9, 12], atol=1e-4)
    np.testing.assert_allclose(acc * np.float32(0.5), [1.5, 3, 4.5, 6], atol=1e-4)


def test_vector_math_int8_with_stored_scale():
    """STT/generation/attention/PagedAttentionVectorMathTest.java:41-59."""
    q = np.array([1, 2, 3], np.float32)
    key = np.array([2, -4, 6], np.int8)
    value = np.array([4, 6, -8], np.int8)
    s = O.score(O.INT8, q, key, scale_seg=np.array([0.5], np.float32), dim=3, scale=2.0)
    assert abs(s - 12.0) <= 1e-4
    acc = O.update(O.INT8, np.array([2, 4, 6], np.float32), value,
                   scale_seg=np.array([0.25], np.float32), prev=0.5, cur=2.0)
    np.testing.assert_allclose(acc, [3, 5, -1], atol=1e-4)


def test_vector_math_int4_with_stored_scale():
    """STT/generation/attention/PagedAttentionVectorMathTest.java:61-87."""
    one = np.float32(2.0) / np.float32(7.0)
    q = np.ones(4, np.float32)
    key = np.zeros(2, np.uint8)
    value = np.zeros(2, np.uint8)
    ks = np.zeros(1, np.float32)
    vs = np.zeros(1, np.float32)
    O.write_vector(O.INT4, np.array([-2, 0, 2, -one], np.float32), key, 0, ks, 0)
    O.write_vector(O.INT4, np.array([2, -2, 0, one], np.float32), value, 0, vs, 0)
    s = O.score(O.INT4, q, key, scale_seg=ks, dim=4, scale=3.0)
    assert abs(s - (-3.0 * one)) <= 1e-4
    acc = O.update(O.INT4, np.zeros(4, np.float32), value, scale_seg=vs, prev=0.0, cur=1.0)
    np.testing.assert_allclose(acc, [2, -2, 0, one], atol=1e-4)


def test_attention_fp32_vector_math():
    """STT/generation/attention/AttentionFp32VectorMathTest.java:20-37 (5 lanes' worth: a tail)."""
    q = np.array([1, 2, 3, 4, 5], np.float32)
    key = np.array([0.5, -1, 2, 1, -2], np.float32)
    value = np.array([10, 20, 30, 40, 50], np.float32)
    for lanes in (1, 2, 4, 8, 16):
        assert abs(O.fp32_dot(q, key, lanes) - (-1.5)) <= 1e-4
    acc = O.fp32_update(np.array([1, 2, 3, 4, 5], np.float32), value, 0.5, 0.25)
    np.testing.assert_allclose(acc, [3, 6, 9, 12, 15], atol=1e-4)


# --------------------------------------------------- PagedKvCacheQuantization

def test_int8_round_trip():
    """STT/generation/attention/PagedKvCacheQuantizationTest.java:20-35."""
    src = np.array([-2, 0, 2], np.float32)
    qb = np.zeros(3, np.int8)
    sc = np.zeros(1, np.float32)
    O.write_vector(O.INT8, src, qb, 0, sc, 0)
    assert list(qb) == [-127, 0, 127]
    back = O.read_vector(O.INT8, qb, sc, 0, 0, 3)
    np.testing.assert_allclose(back, src, atol=1e-4)


def test_int4_nibbles_and_round_trip():
    """STT/generation/attention/PagedKvCacheQuantizationTest.java:37-59: nibbles -7, 0, 7, -1."""
    one = np.float32(2.0) / np.float32(7.0)
    src = np.array([-2, 0, 2, -one], np.float32)
    qb = np.zeros(2, np.uint8)
    sc = np.zeros(1, np.float32)
    O.write_vector(O.INT4, src, qb, 0, sc, 0)
    vals = [(int(qb[e >> 1]) >> (4 * (e & 1)) & 0xF) - 8 for e in range(4)]
    assert vals == [-7, 0, 7, -1]
    back = O.read_vector(O.INT4, qb, sc, 0, 0, 4)
    np.testing.assert_allclose(back, src, atol=1e-4)


def test_zero_vector_scale_is_one():
    """PagedKvCacheQuantization.vectorScale: absmax 0 -> scale 1.0 (:105)."""
    qb = np.zeros(4, np.int8)
    sc = np.zeros(1, np.float32)
    O.write_vector(O.INT8, np.zeros(4, np.float32), qb, 0, sc, 0)
    assert sc[0] == 1.0 and not qb.any()


def test_java_round_ties_toward_positive_infinity():
    """Math.round(float) as used by quantizeVectorToInt8 (:75)."""
    assert O.java_round(2.5) == 3
    assert O.java_round(-2.5) == -2
    assert O.java_round(-0.5) == 0
    assert O.java_round(0.49999997) == 0
    assert O.java_round(-126.5) == -126
    assert O.java_round(float("nan")) == 0


# ------------------------------------------------------- AttentionOnlineSoftmax

def test_online_softmax_weights():
    """STT/generation/attention/AttentionOnlineSoftmaxTest.java:15-32."""
    norm, prev, cur, inv = O.softmax_observe([2.0])
    assert abs(prev - 0.0) <= 1e-4 and abs(cur - 1.0) <= 1e-4 and abs(inv - 1.0) <= 1e-4
    norm, prev, cur, inv = O.softmax_observe([2.0, 4.0])
    pw = math.exp(-2.0)
    assert abs(prev - pw) <= 1e-4
    assert abs(cur - 1.0) <= 1e-4
    assert abs(inv - 1.0 / (pw + 1.0)) <= 1e-4


# ------------------------------------------------------------- layout / context

def test_layout_offsets():
    """STT/generation/attention/PagedKvCacheLayoutTest.java:16-38 (BlockManager [H][BS][D])."""
    H, D, BS = 2, 4, 16
    head_stride, tok_stride, scale_stride = BS * D, D, BS
    assert 19 % BS == 3
    assert 1 * head_stride + 3 * tok_stride == 76
    assert (1 * head_stride + 3 * tok_stride) * 4 == 304
    assert 1 * scale_stride + 3 == 19
    assert (5 * H + 1) * D == 44                              # tokenMajorElement(5, 1)
    assert 2 * (H * BS * D) + 1 * (BS * D) + 3 * D == 332     # blockMajorElement(2, 1, 3)
    assert H * BS * D == 128


def test_int4_block_bytes():
    """STT/generation/kv/KVCacheAllocationTest.java:44-71: 16 tokens x 64 dims int4 = 512 B."""
    assert O.block_bytes(O.INT4, 1, 16, 64) == 512
    assert O.block_bytes(O.INT8, 1, 16, 64) == 1024
    assert O.block_bytes(O.FP32, 1, 16, 64) == 4096


def _single_block_case(Hq, Hkv, D, BS, total, seed=0):
    rng = np.random.default_rng(seed)
    nb = (total + BS - 1) // BS
    k = rng.standard_normal((nb, Hkv, BS, D)).astype(np.float32)
    v = rng.standard_normal((nb, Hkv, BS, D)).astype(np.float32)
    q = rng.standard_normal((1, 1, Hq, D)).astype(np.float32)
    bt = np.arange(nb, dtype=np.int32)[None]
    return q, k, v, bt


def test_gqa_head_map_and_window():
    """STT/generation/attention/PagedAttentionVectorContextTest.java:20-60.

    Hq=4, Hkv=2: q-head 3 reads kv-head 1 (qHead / (Hq/Hkv)); a window of 4 at
    position 9 starts at 6.  Checked through the oracle's outputs: q-head 3 equals
    an MHA run on kv-head 1 alone, and a windowed run equals a run over the last
    four tokens only.
    """
    Hq, Hkv, D, BS, total = 4, 2, 5, 8, 10
    q, k, v, bt = _single_block_case(Hq, Hkv, D, BS, total)
    ctx = np.array([total], np.int32)
    out = O.a2_compute(q, k, v, bt, ctx, 0.25, num_kv_heads=Hkv, block_size=BS)
    single = O.a2_compute(q[:, :, 3:4], np.ascontiguousarray(k[:, 1:2]),
                          np.ascontiguousarray(v[:, 1:2]), bt, ctx, 0.25, num_kv_heads=1,
                          block_size=BS)
    np.testing.assert_array_equal(out[0, 0, 3], single[0, 0, 0])

    win = O.a2_compute(q, k, v, bt, ctx, 0.25, num_kv_heads=Hkv, block_size=BS, sliding_window=4)
    # Tokens 6..9 only: shift them to a fresh single block.
    k2 = np.zeros((1, Hkv, BS, D), np.float32)
    v2 = np.zeros((1, Hkv, BS, D), np.float32)
    for j, t in enumerate(range(6, 10)):
        k2[0, :, j] = k[t // BS, :, t % BS]
        v2[0, :, j] = v[t // BS, :, t % BS]
    ref = O.a2_compute(q, k2, v2, np.zeros((1, 1), np.int32), np.array([4], np.int32), 0.25,
                       num_kv_heads=Hkv, block_size=BS)
    np.testing.assert_allclose(win, ref, rtol=1e-6, atol=1e-7)


def test_a1_and_a2_agree_on_mha():
    """The two reference CPU paths compute the same attention (fp32, MHA)."""
    rng = np.random.default_rng(7)
    S, H, D, BS, NB = 3, 4, 16, 4, 40
    ctx = np.array([1, 13, 37], np.int32)
    maxB = 10
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.full((S, maxB), -1, np.int32)
    off = 0
    for s in range(S):
        n = (ctx[s] + BS - 1) // BS
        bt[s, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((S, H, D)).astype(np.float32)
    k = rng.standard_normal((NB, H, BS, D)).astype(np.float32)
    v = rng.standard_normal((NB, H, BS, D)).astype(np.float32)
    a1 = O.a1_execute(q, k, v, bt, ctx, 0.25)
    a2 = O.a2_compute(q, k, v, bt, ctx, 0.25, num_kv_heads=H, block_size=BS)[:, 0]
    np.testing.assert_allclose(a1, a2, rtol=1e-5, atol=1e-6)


def test_empty_context_gives_zeros():
    """contextLen 0: a1 writes acc = 0; a2 writes 0 * 1/(0 + 1e-9) = 0."""
    q = np.ones((1, 2, 4), np.float32)
    k = np.ones((1, 2, 4, 4), np.float32)
    bt = np.zeros((1, 1), np.int32)
    ctx = np.zeros(1, np.int32)
    assert not O.a1_execute(q, k, k, bt, ctx, 1.0).any()
    assert not O.a2_compute(q, k, k, bt, ctx, 1.0, num_kv_heads=2, block_size=4).any()


def test_update_cache_then_gather_round_trip():
    """PagedKvCacheIOTest.java:29-46: a written token reads back; unused table entries skipped."""
    BS, Hkv, D = 16, 1, 2
    k_slab = np.zeros((2, Hkv, BS, D), np.float32)
    v_slab = np.zeros((2, Hkv, BS, D), np.float32)
    bt = np.array([[1, -1]], np.int32)
    rc = O.update_cache(np.array([[[1.0, 2.0]]]), np.array([[[101.0, 102.0]]]), [0], bt,
                        storage=O.FP32, k_slab=k_slab, v_slab=v_slab, block_size=BS)
    assert rc == 0
    np.testing.assert_array_equal(k_slab[1, 0, 0], [1, 2])
    np.testing.assert_array_equal(v_slab[1, 0, 0], [101, 102])
    assert O.update_cache(np.zeros((1, 1, 2)), np.zeros((1, 1, 2)), [16], bt, storage=O.FP32,
                          k_slab=k_slab, v_slab=v_slab, block_size=BS) == -1


def test_migrate_copies_remapped_slices():
    """PD/PrefillDecodeDisaggService.java:415-429 over PhysicalBlockPool offsets."""
    L, bpb, nb = 3, 64, 6
    rng = np.random.default_rng(1)
    k = rng.integers(0, 255, nb * L * bpb, dtype=np.uint8)
    v = rng.integers(0, 255, nb * L * bpb, dtype=np.uint8)
    k0, v0 = k.copy(), v.copy()
    copied = O.migrate(k, v, k, v, [0, 2], [5, 3], L, bpb)
    assert copied == 2 * 2 * L * bpb
    kb = k.reshape(nb, L * bpb)
    vb = v.reshape(nb, L * bpb)
    np.testing.assert_array_equal(kb[5], k0.reshape(nb, -1)[0])
    np.testing.assert_array_equal(kb[3], k0.reshape(nb, -1)[2])
    np.testing.assert_array_equal(vb[5], v0.reshape(nb, -1)[0])
    np.testing.assert_array_equal(kb[1], k0.reshape(nb, -1)[1])


def test_bf16_helpers_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.5, 0.0], np.float32)
    r = O.round_bf16(x)
    np.testing.assert_array_equal(r, [1.0, 1.0, 1.015625, -3.5, 0.0])


@pytest.mark.parametrize("threads", [2, 4])
def test_parallel_oracle_matches_serial(threads):
    rng = np.random.default_rng(3)
    S, Hq, Hkv, D, BS, NB = 4, 8, 2, 32, 16, 64
    ctx = np.array([5, 100, 250, 16], np.int32)
    maxB = 16
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.zeros((S, maxB), np.int32)
    off = 0
    for s in range(S):
        n = (ctx[s] + BS - 1) // BS
        bt[s, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((S, 1, Hq, D)).astype(np.float32)
    k = rng.standard_normal((NB, Hkv, BS, D)).astype(np.float32)
    v = rng.standard_normal((NB, Hkv, BS, D)).astype(np.float32)
    a = O.a2_compute(q, k, v, bt, ctx, 0.2, num_kv_heads=Hkv, block_size=BS)
    b = O.a2_compute(q, k, v, bt, ctx, 0.2, num_kv_heads=Hkv, block_size=BS, threads=threads)
    np.testing.assert_array_equal(a, b)
