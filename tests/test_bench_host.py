"""Host-side pieces of bench.py that shape its JSON line, checked on the CPU: the
config-1 sweep, the algorithmic bytes, the launch count it claims, and the ncu traffic
figure it reads from profiles/ for the roofline kernel."""
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


def test_launch_count_rule():
    # split-mode launches stage activations in a prep kernel; the two LM-head GEMVs run
    # in whole mode and stage in-kernel
    per = {(n, k): bench.launches_per_gemv(t, n, k) for _, t, n, k in bench.sweep()}
    assert per[(151936, 896)] == 1
    assert all(v == 2 for (n, _), v in per.items() if n != 151936)
    assert sum(bench.launches_per_gemv(t, n, k) for _, t, n, k in bench.sweep()) == 26


def test_roofline_traffic_from_profiles():
    # the bench's roofline kernel reads its DRAM bytes per launch from the ncu summary
    assert bench.profile_traffic("qgemv_q8_0_151936x896_m1") == 148566784.0
    assert bench.profile_traffic("no_such_kernel") is None
