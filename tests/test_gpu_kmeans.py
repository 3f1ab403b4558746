"""GPU: K-means assignment with the argmin fused into the skinny GEMM."""
from __future__ import annotations

import pytest
import torch

from oracle import oracle
from tensorcore_gemm import kmeans

pytestmark = pytest.mark.gpu


# K <= 128 runs the 16-warp epilogue, K > 128 the 8-warp one.
@pytest.mark.parametrize("M,N,K", [(32768, 1024, 256), (16384, 256, 256), (1000, 300, 64), (129, 5, 40),
                                   (65536, 4096, 128), (4096, 1000, 128), (777, 333, 96), (5000, 700, 200)])
@pytest.mark.parametrize("kn", [False, True])
def test_assign_matches_fp64_argmin(cuda_device, native_lib, M, N, K, kn):
    X, C = oracle.make_inputs(M, N, K, dist="normal", seed_a=M, seed_b=N)   # C: K x N
    X, C = X.to(cuda_device), C.to(cuda_device)
    cent = C if kn else C.t().contiguous()
    idx, score = kmeans.assign(X, cent, centroids_kn=kn, return_scores=True)
    torch.cuda.synchronize()
    Xd, Cd = X.double(), C.double()
    ref = (Cd * Cd).sum(0)[None, :] - 2.0 * (Xd @ Cd)                   # M x N scores
    best = ref.min(1)
    got = ref.gather(1, idx.long()[:, None])[:, 0]
    # fp32 accumulation: a near-tie may resolve either way, never by more than the GEMM bound.
    tol = 2e-3 * K ** 0.5 * (2.0 * (Xd @ Cd)).pow(2).mean().sqrt().item()
    assert (got - best.values).max().item() <= tol
    assert (idx.long() == best.indices).double().mean().item() >= 0.99
    assert (score.double() - got).abs().max().item() <= tol
    assert int(idx.min()) >= 0 and int(idx.max()) < N


def test_assign_ties_go_to_smaller_index(cuda_device, native_lib):
    X = torch.ones((256, 64), dtype=torch.float16, device=cuda_device)
    cent = torch.zeros((600, 64), dtype=torch.float16, device=cuda_device)
    cent[100] = 1.0
    cent[450] = 1.0                                          # same score as 100, in another N slice
    idx = kmeans.assign(X, cent)
    assert torch.all(idx == 100)


@pytest.mark.parametrize("K", [64, 256])
def test_assign_ties_within_and_across_chunks(cuda_device, native_lib, K):
    """Equal best scores in both 32-column halves of one 64-column chunk, and
    in two chunks of the same 256-column slice: the smallest index wins with
    either epilogue (K = 64: 16 warps, K = 256: 8 warps)."""
    X = torch.ones((512, K), dtype=torch.float16, device=cuda_device)
    cent = torch.zeros((300, K), dtype=torch.float16, device=cuda_device)
    for j in (40, 10, 200, 75):
        cent[j] = 1.0
    idx, score = kmeans.assign(X, cent, return_scores=True)
    assert torch.all(idx == 10)
    assert torch.all(score == -float(K))


def test_assign_rejects_long_k(cuda_device, native_lib):
    X = torch.zeros((128, 512), dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError):
        kmeans.assign(X, torch.zeros((16, 512), dtype=torch.float16, device=cuda_device))
