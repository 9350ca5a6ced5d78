"""Host-side accounting of bench.py (no GPU): the algorithmic bytes of the
plaintext-product passes and the NVLink bytes of the input-broadcast
collectives, against hand counts."""
import bench
from comp390project_b200 import matmul

N = 1 << 16
U = 8 * N


def test_mac_alg_bytes_config5():
    lay = matmul.layout(N // 2, 128, 768, 768)
    # 3 outputs x 4 passes of (48 ciphertexts x 2 polys + 4 x 48 diagonals + 4 x 2 outputs)
    assert bench.mac_alg_bytes(lay, 0, 16, 35, N) == 3 * 4 * (96 + 192 + 8) * 35 * U
    # a 2-GPU half: giant steps 8..15, 2 passes per output
    assert bench.mac_alg_bytes(lay, 8, 16, 35, N) == 3 * 2 * (96 + 192 + 8) * 35 * U


def test_mac_alg_bytes_counts_accumulating_passes():
    lay = matmul.layout(2048, 32, 128, 128, n_baby=64)   # 128 terms: two passes of 64
    want = 2 * ((2 * 64 + 64 + 2) + (2 * 64 + 64 + 2 + 2)) * 7 * 8 * 4096
    assert bench.mac_alg_bytes(lay, 0, 1, 7, 4096) == want


def test_collective_roofline_bytes():
    prof = {"collective": (1.0, 8)}
    r8 = bench.collective_roofline(prof, 4, 35, 5, 8, N)
    # 7 peers x (ceil(35/8) = 5 input limbs + 2 polys x 1 P limb)
    assert r8["bytes_received_per_ks"] == 7 * (5 + 2) * U
    r2 = bench.collective_roofline(prof, 4, 35, 5, 2, N)
    # P limbs 35..39 on ranks 1,0,1,0,1: rank 1 owns 3
    assert r2["bytes_received_per_ks"] == 1 * (18 + 2 * 3) * U
    assert abs(r2["frac"] - r2["achieved"] / bench.NVLINK_GBS) < 1e-12
    assert bench.collective_roofline(prof, 4, 35, 5, 1, N) is None
    assert bench.collective_roofline({}, 4, 35, 5, 8, N) is None
