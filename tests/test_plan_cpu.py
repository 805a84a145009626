"""The GEMM's host-side planning (b2g_plan_gemm) on the CPU: what b2g_gemm launches
for the BASELINE configurations on a 148-SM B200, invariants over random
descriptors, and the status codes of descriptors it refuses.  b2g_gemm itself
calls the same planning function, so these are the launch decisions."""
import numpy as np
import pytest

import b2g


def plan(fmt, M, N, K, **kw):
    return b2g.plan_gemm(fmt, M, N, K, **kw)


def test_cfg2_e4m3_8192():
    # two 128-row A sub-tiles per CTA: each pair issues two 256 x 256 MMAs per K step
    # into a 512 x 256 tile (7 waves of 512 tiles against 14 of 1024 256-row tiles)
    p = plan(b2g.FMT_E4M3, 8192, 8192, 8192, cta_group=2, tile_n=256)
    assert (p["variant"], p["cta_group"], p["tile_m"], p["tile_n"], p["m_sub"]) == (0, 2, 512, 256, 2)
    assert p["stages"] == 4 and p["smem_bytes"] <= 227 * 1024 and p["tmem_columns"] == 512
    assert (p["num_m_tiles"], p["num_n_tiles"], p["k_blocks"]) == (16, 32, 64)
    # one accumulator buffer: no split tail
    assert (p["tail_split"], p["units"], p["clusters"], p["threads"]) == (1, 512, 74, 320)
    # one sub-tile (256 x 256 pair tiles, double-buffered accumulator) on request
    p = plan(b2g.FMT_E4M3, 8192, 8192, 8192, cta_group=2, tile_n=256, m_sub=1)
    assert (p["tile_m"], p["m_sub"], p["stages"], p["tmem_columns"]) == (256, 1, 7, 512)
    assert (p["num_m_tiles"], p["num_n_tiles"], p["k_blocks"]) == (32, 32, 64)
    # 1024 tiles on 74 clusters: the last wave holds 62 tiles, too many to split
    assert (p["tail_split"], p["units"], p["clusters"], p["threads"]) == (1, 1024, 74, 192)


def test_default_tile_n_counts_whole_waves():
    # 4096^3 bf16 on 74 pairs: 4 waves of 256 columns cost more than 5 of 192
    p = plan(b2g.FMT_BF16, 4096, 4096, 4096)
    assert (p["cta_group"], p["tile_n"], p["num_n_tiles"], p["tail_split"]) == (2, 192, 22, 1)
    # 8192^3: 14 waves of 256 against 19 of 192 -> 256
    assert plan(b2g.FMT_E4M3, 8192, 8192, 8192)["tile_n"] == 256
    # fewer clusters change the count: 4096^3 on 64 pairs is 4 waves of 256 against 6 of 192
    assert plan(b2g.FMT_BF16, 4096, 4096, 4096, max_clusters=64)["tile_n"] == 256
    # block-scaled and sparse keep their 224-column default
    assert plan(b2g.FMT_NVFP4, 4096, 4096, 4096)["tile_n"] == 224


def test_cfg1_bf16_4096_splits_its_tail():
    p = plan(b2g.FMT_BF16, 4096, 4096, 4096, cta_group=2, tile_n=256)
    assert p["num_m_tiles"] * p["num_n_tiles"] == 256 and p["k_blocks"] == 64
    # 3 full waves of 74 clusters (222 tiles), 34 tail tiles cut in 2 K halves
    assert (p["tail_start"], p["tail_split"], p["units"], p["clusters"]) == (222, 2, 290, 74)


def test_cfg3_sparse_two_subtiles():
    p = plan(b2g.FMT_BF16, 8192, 8192, 16384, sparse=1, cta_group=2)
    assert (p["variant"], p["m_sub"], p["tile_m"], p["tile_n"], p["threads"]) == (1, 2, 512, 224, 320)
    assert p["stages"] == 3 and p["tmem_columns"] == 512
    assert (p["num_m_tiles"], p["num_n_tiles"], p["k_blocks"]) == (16, 37, 128)
    assert p["tail_split"] == 1 and p["units"] == 592 and p["clusters"] == 74


@pytest.mark.parametrize("fmt,variant,K", [(b2g.FMT_NVFP4, 2, 16384), (b2g.FMT_MXF8, 3, 8192),
                                           (b2g.FMT_MXF4, 4, 16384)])
def test_block_scaled_defaults(fmt, variant, K):
    p = plan(fmt, 16384, 16384, K, cta_group=2)
    assert (p["variant"], p["m_sub"], p["tile_n"], p["tmem_columns"]) == (variant, 2, 224, 512)
    assert 2 <= p["stages"] <= 8 and p["smem_bytes"] <= 227 * 1024


def test_max_clusters_caps_the_grid_and_resplits():
    p = plan(b2g.FMT_BF16, 4096, 4096, 4096, cta_group=2, tile_n=256, max_clusters=60)
    assert p["clusters"] == 60
    # 256 tiles on 60 clusters: 16 in the last wave -> 3 K splits
    assert (p["tail_start"], p["tail_split"]) == (240, 3)


def test_split_tail_off_and_forced():
    off = plan(b2g.FMT_BF16, 4096, 4096, 4096, cta_group=2, tile_n=256, split_tail=1)
    assert off["tail_split"] == 1 and off["units"] == 256
    two = plan(b2g.FMT_BF16, 1024, 1024, 2048, cta_group=2, tile_n=256, max_ctas=10, split_tail=2)
    assert two["tail_split"] == 2 and two["tail_start"] == 15


def test_plan_invariants_random():
    rng = np.random.default_rng(5)
    fmts = [b2g.FMT_BF16, b2g.FMT_E4M3, b2g.FMT_NVFP4, b2g.FMT_MXF8, b2g.FMT_MXF4, b2g.FMT_S8,
            b2g.FMT_TF32, b2g.FMT_E5M2]
    checked = 0
    for _ in range(400):
        fmt = int(rng.choice(fmts))
        sparse = int(fmt == b2g.FMT_BF16 and rng.random() < 0.3)
        M, N = int(rng.integers(1, 20000)), int(rng.integers(1, 20000))
        K = int(rng.integers(1, 600)) * 32
        kw = dict(cta_group=int(rng.choice([0, 1, 2])), tile_n=int(rng.choice([0, 64, 128, 224, 256])),
                  split_tail=int(rng.integers(0, 5)), max_ctas=int(rng.choice([0, 8, 40, 148])))
        if fmt in (b2g.FMT_NVFP4, b2g.FMT_MXF8, b2g.FMT_MXF4) or sparse:
            kw["m_sub"] = int(rng.integers(0, 3))
        sm = int(rng.choice([148, 132, 8]))
        try:
            p = plan(fmt, M, N, K, sparse=sparse, sm_count=sm, **kw)
        except b2g.B2GError as e:
            assert e.status in (1, 4)
            continue
        checked += 1
        cg = p["cta_group"]
        assert p["tile_m"] == 128 * p["m_sub"] * cg
        assert 2 <= p["stages"] <= 8 and p["smem_bytes"] <= 227 * 1024
        t = p["tmem_columns"]
        assert 32 <= t <= 512 and t & (t - 1) == 0
        tiles = p["num_m_tiles"] * p["num_n_tiles"]
        assert p["num_m_tiles"] * p["tile_m"] >= M and p["num_n_tiles"] * p["tile_n"] >= N
        assert 1 <= p["tail_split"] <= 4
        if fmt == b2g.FMT_S8:
            assert p["tail_split"] == 1
        if p["tail_split"] > 1:
            assert p["m_sub"] == 1 and p["tail_split"] * 2 <= p["k_blocks"]
            # each cluster of the grid takes at most one tail unit
            assert (tiles - p["tail_start"]) * p["tail_split"] <= p["clusters"]
        assert p["units"] == (p["tail_start"] + (tiles - p["tail_start"]) * p["tail_split"]
                              if p["tail_split"] > 1 else tiles)
        assert 1 <= p["clusters"] <= min(p["units"], sm // cg)
        assert p["threads"] == (320 if p["m_sub"] == 2 else 192)
        # two K atoms per slot only for narrow dense SS tiles with a 4-deep ring
        assert p["k_atoms"] in (1, 2)
        if p["k_atoms"] == 2:
            assert p["variant"] == 0 and p["m_sub"] == 1 and p["tile_n"] <= 128
            assert p["stages"] >= 4 or kw.get("stages", 0) not in (0, None)
    assert checked > 200


@pytest.mark.parametrize("fmt,M,N,K,kw,status", [
    (99, 256, 256, 256, {}, 4),                                  # unknown format
    (b2g.FMT_BF16, 256, 256, 256, dict(sparse=1, ab_mode=1), 4),  # TS with sparse
    (b2g.FMT_NVFP4, 256, 256, 256, dict(ab_mode=1), 4),          # TS with block scales
    (b2g.FMT_BF16, 256, 256, 256, dict(tile_n=48), 1),
    (b2g.FMT_BF16, 256, 256, 256, dict(m_sub=2, ab_mode=1), 4),  # dense two sub-tiles: SS only
    (b2g.FMT_BF16, 256, 256, 256, dict(stages=9), 1),
    (b2g.FMT_MXF8, 256, 256, 48, {}, 1),                         # MX: K % 32
    (b2g.FMT_BF16, 256, 256, 256, dict(split_tail=5), 1),
    (b2g.FMT_BF16, 256, 256, 256, dict(lda=100), 1),
    (b2g.FMT_NVFP4, 256, 256, 256, dict(tile_n=256), 1),         # no TMEM left for scales
    (b2g.FMT_BF16, 0, 256, 256, {}, 1),
])
def test_refusals(fmt, M, N, K, kw, status):
    with pytest.raises(b2g.B2GError) as e:
        plan(fmt, M, N, K, **kw)
    assert e.value.status == status


def test_s8_never_splits_its_tail():
    # i8 tiles stay whole (s32 partial sums would be added in fp32); tf32 splits
    p = plan(b2g.FMT_S8, 1280, 1024, 2048, cta_group=2, tile_n=256, max_ctas=32)
    assert p["tail_split"] == 1 and p["kind"] == 3
    q = plan(b2g.FMT_TF32, 1280, 1024, 2048, cta_group=2, tile_n=256, max_ctas=32)
    assert q["tail_split"] >= 2 and q["kind"] == 0


@pytest.mark.parametrize("fmt", [b2g.FMT_S8, b2g.FMT_TF32, b2g.FMT_E5M2])
def test_ts_refused_for_the_other_dense_kinds(fmt):
    with pytest.raises(b2g.B2GError):
        plan(fmt, 256, 256, 256, ab_mode=1)


def test_tf32_k_slot_is_32_elements():
    p = plan(b2g.FMT_TF32, 512, 512, 1000, tile_n=256)
    assert p["k_blocks"] == 32 and p["k_atoms"] == 1  # ceil(1000 / 32)
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_TF32, 512, 512, 1002)  # row stride 4008 bytes: not a multiple of 16


@pytest.mark.parametrize("fmt", [b2g.FMT_E2M1, b2g.FMT_E2M3, b2g.FMT_E3M2])
def test_sub_byte_f8f6f4_plans(fmt):
    # packed fp4 / fp6: 128 elements per ring slot, like fp8
    p = plan(fmt, 8192, 8192, 8192, cta_group=2, tile_n=256, m_sub=1)
    assert (p["kind"], p["k_blocks"], p["stages"]) == (2, 64, 7)
    p = plan(fmt, 8192, 8192, 8192, cta_group=2, tile_n=256)
    assert (p["kind"], p["k_blocks"], p["stages"], p["m_sub"]) == (2, 64, 4, 2)
    for kw in (dict(K=8192 + 64), dict(lda=8192 + 64)):
        K = kw.get("K", 8192)
        with pytest.raises(b2g.B2GError) as e:
            plan(fmt, 8192, 8192, K, lda=kw.get("lda"), ldb=8192 if "lda" in kw else None)
        assert e.value.status == 1


def test_i8_accumulator_range_is_enforced():
    assert plan(b2g.FMT_U8, 256, 256, 33024)["kind"] == 3
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_U8, 256, 256, 33280)
    assert plan(b2g.FMT_S8, 256, 256, 131056)["kind"] == 3
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_S8, 256, 256, 131072)


def test_f16_is_its_own_kind_f16_type():
    p = plan(b2g.FMT_F16, 512, 512, 512)
    assert p["kind"] == 1 and p["k_blocks"] == 8
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_F16, 512, 512, 512, ab_mode=1)  # TS is built for bf16 / e4m3


def test_f8f6f4_type_mixes_and_refusals():
    p = plan(b2g.FMT_E4M3, 512, 512, 1024, b_format=b2g.FMT_E2M1)
    assert (p["kind"], p["k_blocks"]) == (2, 8)
    # B packed fp4: K and ldb multiples of 128; A e4m3 keeps its 16-byte rule
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_E4M3, 512, 512, 1040, b_format=b2g.FMT_E2M1)
    assert plan(b2g.FMT_E4M3, 512, 512, 1024, lda=1040, b_format=b2g.FMT_E2M1)["kind"] == 2
    # no other kind mixes: f16 / bf16 (a mix faults the MMA), i8 s / u8, MX scaled
    for a, b in ((b2g.FMT_BF16, b2g.FMT_F16), (b2g.FMT_S8, b2g.FMT_U8),
                 (b2g.FMT_MXF8, b2g.FMT_E4M3), (b2g.FMT_E4M3, b2g.FMT_TF32)):
        with pytest.raises(b2g.B2GError) as e:
            plan(a, 512, 512, 1024, b_format=b)
        assert e.value.status == 4
    # TS takes no mix
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_E4M3, 512, 512, 1024, b_format=b2g.FMT_E5M2, ab_mode=1)


def test_mx_scale_on_f8f6f4_element_types():
    for f in (b2g.FMT_E4M3, b2g.FMT_E5M2, b2g.FMT_E2M1, b2g.FMT_E2M3, b2g.FMT_E3M2):
        p = plan(f, 4096, 4096, 4096, mx_scale=1)
        assert (p["variant"], p["kind"], p["tile_n"]) == (3, 4, 224)
    p = plan(b2g.FMT_E4M3, 4096, 4096, 4096, mx_scale=1, b_format=b2g.FMT_E2M1)
    assert p["kind"] == 4
    for f in (b2g.FMT_BF16, b2g.FMT_S8, b2g.FMT_TF32, b2g.FMT_NVFP4):
        with pytest.raises(b2g.B2GError) as e:
            plan(f, 512, 512, 512, mx_scale=1)
        assert e.value.status == 4
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_E4M3, 512, 512, 512, mx_scale=1, ab_mode=1)


def test_dense_two_subtiles_plan():
    for tn in (224, 256):
        p = plan(b2g.FMT_E4M3, 8192, 8192, 8192, cta_group=2, tile_n=tn, m_sub=2)
        assert (p["tile_m"], p["m_sub"], p["threads"], p["tmem_columns"], p["tail_split"]) == (512, 2, 320, 512, 1)
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_E4M3, 8192, 8192, 8192, cta_group=2, m_sub=2, tile_n=224, ab_mode=1)
    for f in (b2g.FMT_S8, b2g.FMT_TF32):
        with pytest.raises(b2g.B2GError):
            plan(f, 8192, 8192, 8192, cta_group=2, tile_n=224, m_sub=2)
    # default: two sub-tiles on 256-column pair tiles with K >= 8192, where at least 4
    # waves of 512-row tiles take no longer than twice as many of 256-row tiles
    assert plan(b2g.FMT_E4M3, 8192, 8192, 8192)["m_sub"] == 2
    assert plan(b2g.FMT_BF16, 8192, 8192, 8192)["m_sub"] == 2
    assert plan(b2g.FMT_BF16, 16384, 16384, 16384)["m_sub"] == 2
    assert plan(b2g.FMT_BF16, 4096, 4096, 4096)["m_sub"] == 1          # 192-column tiles
    assert plan(b2g.FMT_E4M3, 8192, 8192, 4096)["m_sub"] == 1          # short K
    assert plan(b2g.FMT_E4M3, 4096, 4096, 8192, tile_n=256)["m_sub"] == 1  # 2 waves
    assert plan(b2g.FMT_E4M3, 8192, 8192, 8192, tile_n=224)["m_sub"] == 1
    assert plan(b2g.FMT_E4M3, 8192, 8192, 8192, cta_group=1)["m_sub"] == 1
    assert plan(b2g.FMT_E4M3, 8192, 8192, 8192, ab_mode=1)["m_sub"] == 1  # TS
    assert plan(b2g.FMT_S8, 8192, 8192, 8192)["m_sub"] == 1
    # 2560 rows: 5 waves of 320 256-row tiles against 3 (= 6) of 160 512-row ones
    assert plan(b2g.FMT_E4M3, 2560, 8192, 8192, tile_n=256)["m_sub"] == 1


def test_two_k_atoms_for_narrow_dense_tiles():
    # two 128-byte K atoms per slot where the ring keeps 4 stages of them (MMA N <= 128)
    got = {(cg, tn): plan(b2g.FMT_BF16, 8192, 8192, 8192, cta_group=cg, tile_n=tn)
           for cg, tn in ((1, 64), (1, 128), (2, 128), (2, 192), (2, 256))}
    assert {k: (p["k_atoms"], p["stages"]) for k, p in got.items()} == {
        (1, 64): (2, 4), (1, 128): (1, 7), (2, 128): (2, 4), (2, 192): (1, 8), (2, 256): (1, 4)}
    assert got[(2, 128)]["k_blocks"] == 8192 // 128 and got[(2, 256)]["k_blocks"] == 8192 // 64
    # not for sparse, block-scaled, TS or two sub-tiles; cfg1 keeps one atom
    assert plan(b2g.FMT_BF16, 8192, 8192, 8192, sparse=1, tile_n=128)["k_atoms"] == 1
    assert plan(b2g.FMT_MXF8, 8192, 8192, 8192, tile_n=128)["k_atoms"] == 1
    assert plan(b2g.FMT_BF16, 8192, 8192, 8192, tile_n=128, ab_mode=1)["k_atoms"] == 1
    assert plan(b2g.FMT_BF16, 4096, 4096, 4096)["k_atoms"] == 1


def test_weight_stationary_plans_and_refusals():
    # tcgen05.mma.ws{.sp}: cta_group 1, 128-row tiles, N 64 / 128 / 256, one K atom
    p = plan(b2g.FMT_BF16, 8192, 8192, 8192, instruction=1)
    assert (p["instruction"], p["cta_group"], p["tile_m"], p["tile_n"], p["k_atoms"]) == (
        1, 1, 128, 256, 1)
    assert plan(b2g.FMT_BF16, 8192, 8192, 8192)["instruction"] == 0
    p = plan(b2g.FMT_BF16, 8192, 8192, 8192, sparse=1, instruction=1)
    assert (p["instruction"], p["m_sub"], p["tile_n"]) == (1, 1, 128)
    assert plan(b2g.FMT_S8, 512, 100, 512, instruction=1)["tile_n"] == 128
    assert plan(b2g.FMT_TF32, 512, 64, 512, instruction=1)["tile_n"] == 64
    assert plan(b2g.FMT_BF16, 8192, 8192, 8192, tile_n=64, instruction=1)["k_atoms"] == 1
    for fmt, kw in ((b2g.FMT_BF16, dict(cta_group=2)), (b2g.FMT_BF16, dict(tile_n=192)),
                    (b2g.FMT_BF16, dict(ab_mode=1)), (b2g.FMT_BF16, dict(m_sub=2)),
                    (b2g.FMT_NVFP4, {}), (b2g.FMT_MXF8, {}), (b2g.FMT_E4M3, dict(mx_scale=1)),
                    (b2g.FMT_BF16, dict(instruction=2))):
        with pytest.raises(b2g.B2GError):
            plan(fmt, 8192, 8192, 8192, **{"instruction": 1, **kw})


def test_sparse_mx_plans_and_refusals():
    # 2:4-sparse A on kind::mxf8f6f4: variant 5, 256 dense K per ring slot, one sub-tile
    for f, kw in ((b2g.FMT_E4M3, dict(mx_scale=1)), (b2g.FMT_E5M2, dict(mx_scale=1)),
                  (b2g.FMT_MXF8, {})):
        p = plan(f, 8192, 8192, 16384, sparse=1, **kw)
        assert (p["variant"], p["kind"], p["m_sub"], p["tile_n"]) == (5, 4, 1, 224)
        assert p["k_blocks"] == 16384 // 256 and p["tmem_columns"] == 512
    assert plan(b2g.FMT_MXF8, 8192, 8192, 8192, sparse=1, m_sub=2, tile_n=192)["m_sub"] == 2
    with pytest.raises(b2g.B2GError):  # one scale per 64 dense K
        plan(b2g.FMT_MXF8, 8192, 8192, 8224, sparse=1)
    for f, kw in ((b2g.FMT_MXF8, dict(m_sub=2, tile_n=224)), (b2g.FMT_E2M1, dict(mx_scale=1)),
                  (b2g.FMT_MXF8, dict(instruction=1))):
        with pytest.raises(b2g.B2GError):
            plan(f, 8192, 8192, 8192, sparse=1, **kw)


def test_sparse_sub_byte_plans_and_refusals():
    # 2:4-sparse fp4 / fp6 on kind::f8f6f4: the 8-bit sparse slot (256 dense K)
    for f in (b2g.FMT_E2M1, b2g.FMT_E2M3, b2g.FMT_E3M2):
        p = plan(f, 8192, 8192, 16384, sparse=1)
        assert (p["variant"], p["kind"], p["k_blocks"]) == (1, 2, 16384 // 256)
        with pytest.raises(b2g.B2GError):  # the compressed row in whole 128-element boxes
            plan(f, 512, 512, 384, sparse=1)
    p = plan(b2g.FMT_E2M1, 4096, 4096, 4096, sparse=1, b_format=b2g.FMT_E4M3)
    assert p["variant"] == 1
    with pytest.raises(b2g.B2GError):  # no sparse MX on the sub-byte types
        plan(b2g.FMT_E2M1, 4096, 4096, 4096, sparse=1, mx_scale=1)


def test_sparse_mxf4_pairs_plan():
    # 4:8 in pairs on kind::mxf4: 512 dense K per ring slot, one sub-tile by default
    p = plan(b2g.FMT_MXF4, 8192, 8192, 16384, sparse=1)
    assert (p["variant"], p["kind"], p["m_sub"], p["tile_n"]) == (6, 5, 2, 192)
    assert p["k_blocks"] == 16384 // 512 and p["tmem_columns"] == 512
    assert plan(b2g.FMT_MXF4, 8192, 8192, 16384, sparse=1, m_sub=1, tile_n=224)["m_sub"] == 1
    with pytest.raises(b2g.B2GError):
        plan(b2g.FMT_MXF4, 8192, 8192, 8224, sparse=1)  # metadata words of 64 elements


def test_sparse_nvfp4_pairs_plan():
    # 4:8 in pairs on kind::mxf4nvf4 block16: 512 dense K per slot, 192-column tiles
    p = plan(b2g.FMT_NVFP4, 16384, 16384, 16384, sparse=1)
    assert (p["variant"], p["kind"], p["m_sub"], p["tile_n"]) == (7, 6, 2, 192)
    assert p["k_blocks"] == 16384 // 512 and p["tmem_columns"] == 512
    assert plan(b2g.FMT_NVFP4, 16384, 16384, 16384, sparse=1, m_sub=1)["tile_m"] == 256
    with pytest.raises(b2g.B2GError):  # TMEM: metadata ring + 48 scale columns
        plan(b2g.FMT_NVFP4, 8192, 8192, 8192, sparse=1, tile_n=224)
