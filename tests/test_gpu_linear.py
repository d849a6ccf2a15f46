"""The dense BF16 projection (qk_linear_bf16) against an FP64 product of the same BF16
operands: the tcgen05 pass accumulates in FP32 (in its own order) and rounds once to BF16,
so a result lies within one BF16 step of the FP64 value plus the FP32 accumulation error,
bounded by a few units of 2^-24 times the sum of |x| |w| over K."""

import numpy as np
import pytest

from oracle.precision import bf16_round
from util import bf16_tensor, to_f32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,N", [(1, 2048, 9216), (8, 4096, 2048), (64, 2048, 9216), (64, 4096, 2048),
                                   (37, 128, 300), (256, 256, 128), (3, 64, 129)])
def test_linear_bf16_matches_fp64(cuda_device, M, K, N):
    import torch

    from qk_b200.packed import linear_bf16, linear_workspace

    rng = np.random.default_rng(M * 131 + N)
    x = bf16_round(rng.normal(size=(M, K)).astype(np.float32))
    w = bf16_round(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    xd, wd = bf16_tensor(x, cuda_device), bf16_tensor(w, cuda_device)
    ws = linear_workspace(M, K, N, cuda_device)
    first = linear_bf16(xd, wd, workspace=ws)
    second = linear_bf16(xd, wd, workspace=ws)  # the workspace is left ready: same bits again
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))
    got = to_f32(first)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)  # one BF16 step at |ref|
    acc = 2.0 ** -20 * (np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T)
    assert np.all(np.abs(got - ref) <= ulp + acc), float(np.max(np.abs(got - ref) / (ulp + acc)))
    assert np.mean(got == bf16_round(ref.astype(np.float32))) > 0.9


def test_linear_bf16_rejects_bad_shapes_before_launch(cuda_device):
    import torch

    from qk_b200.packed import linear_bf16

    x = torch.zeros((300, 64), dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros((128, 64), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        linear_bf16(x, w)
    with pytest.raises(ValueError):
        linear_bf16(torch.zeros((4, 100), dtype=torch.bfloat16, device=cuda_device),
                    torch.zeros((128, 100), dtype=torch.bfloat16, device=cuda_device))
