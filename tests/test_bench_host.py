"""Host-side pieces of bench.py that shape its JSON line, checked on the CPU: the
config-3 step's shards and bytes, the config-1 sweep, the algorithmic bytes, and the ncu
traffic figure it reads from profiles/ for a roofline kernel."""
import bench


def test_sweep_points():
    pts = bench.sweep()
    assert len(pts) == 14  # Q4_K / Q6_K cannot take K = 896
    assert ("Q4_K", 12, 151936, 896) not in pts and ("Q8_0", 8, 151936, 896) in pts


def test_algorithmic_bytes():
    # Q4_K 14336 x 4096: 144 bytes per 256 weights, bf16 x in and y out
    assert bench.weight_bytes(12, 14336, 4096) == 14336 * 16 * 144
    assert bench.alg_bytes(12, 14336, 4096) == 14336 * 16 * 144 + 4096 * 2 + 14336 * 2
    # FP8 carries one f32 scale per row
    assert bench.weight_bytes(0, 4096, 4096) == 4096 * 4096 + 4 * 4096


def test_config3_step_bytes_and_shards():
    # one layer at Q4_K_M-style formats: q, k, o, gate, up Q4_K; v, down Q6_K
    layer = (8192 * 8192 + 1024 * 8192 + 8192 * 8192 + 2 * 28672 * 8192) * 144 // 256 \
        + (1024 * 8192 + 8192 * 28672) * 210 // 256
    assert bench.step_weight_bytes(1) == 80 * layer
    assert abs(bench.step_weight_bytes(1) / 1e9 - 43.52) < 0.01
    for world in (2, 4, 8):
        # column shards split N, row shards split K on superblock boundaries
        for _, t, n, k, sp, _ in bench.LAYER_LINEARS:
            ns, ks = bench.shard_shape(n, k, sp, world)
            assert ns * ks * world == n * k and ks % 256 == 0
        assert bench.step_weight_bytes(world) * world == bench.step_weight_bytes(1)


def test_roofline_traffic_from_profiles():
    # the bench's roofline kernel reads its DRAM bytes per launch from the ncu summary
    assert bench.profile_traffic("qgemv_q8_0_151936x896_m1") == 148566784.0
    assert bench.profile_traffic("no_such_kernel") is None
