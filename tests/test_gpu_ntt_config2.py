"""Config 2 on its own prime chain: 128 polynomials x 36 limbs (one 58-bit +
35 x 42-bit primes, all 1 mod 2^17) x N = 2^16, batched forward then inverse
NTT through ks_ntt_forward / ks_ntt_inverse.  Every limb must come back
unchanged (2.4 GB, compared on the device), and the forward transform must
equal the CPU oracle on a sample of (polynomial, limb) pairs that covers the
58-bit prime, 42-bit primes and the first and last polynomial of the batch
(the oracle restates the NTT of Phantom's nwt_2d_radix8_forward_inplace,
paper/code_study.tex:493-506)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SAMPLE = [(0, 0), (0, 1), (1, 35), (37, 17), (64, 0), (100, 34), (127, 35)]


def test_config2_batch128_roundtrip_and_forward_sample(cuda_device):
    from comp390project_b200 import KsContext, gen_primes
    from oracle.oracle import Oracle
    log_n, polys = 16, 128
    q = gen_primes(log_n, [58] + [42] * 35)
    assert len(q) == 36 and all(int(x) % (1 << 17) == 1 for x in q)
    N = 1 << log_n
    ctx = KsContext(log_n, q, [], device=0)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1)
    data = torch.empty((polys, 36, N), dtype=torch.int64, device="cuda")
    for j in range(36):
        data[:, j] = torch.randint(0, int(q[j]), (polys, N), generator=gen, device="cuda",
                                   dtype=torch.int64)
    orig = data.clone()
    sample_in = {pl: data[pl[0], pl[1]].cpu().numpy().view(np.uint64).copy() for pl in SAMPLE}
    ctx.ntt_forward(data, 36, 0, polys)
    torch.cuda.synchronize()
    o = Oracle(log_n, q, [])
    for (pi, j), x in sample_in.items():
        got = data[pi, j].cpu().numpy().view(np.uint64)
        want = o.ntt(x.reshape(1, N), [j])[0]
        assert np.array_equal(got, want), ("forward differs", pi, j)
    # every forward output is a canonical residue of its limb's prime
    qs = torch.tensor([int(x) for x in q], dtype=torch.int64, device="cuda").view(1, 36, 1)
    assert bool(((data >= 0) & (data < qs)).all())
    ctx.ntt_inverse(data, 36, 0, polys)
    torch.cuda.synchronize()
    assert torch.equal(data, orig), "inverse(forward(x)) != x on some limb"
    ctx.close()
