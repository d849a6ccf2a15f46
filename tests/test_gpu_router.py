"""Router top-k on the GPU against the oracle: ids exact, weights within one BF16 ulp."""

import numpy as np
import pytest

from oracle import moe
from util import bf16_tensor, to_f32

pytestmark = pytest.mark.gpu


def _gap_ok(probs, ids_a, ids_b, k):
    """Mismatching ids are only allowed at numerical near-ties of the probabilities."""
    for t in np.nonzero((ids_a != ids_b).any(-1))[0]:
        p = np.sort(probs[t])[::-1]
        assert abs(p[k - 1] - p[k]) < 1e-6 * max(p[0], 1e-30), f"row {t} differs without a tie"


@pytest.mark.parametrize("T,E,k", [(8, 64, 4), (64, 512, 10), (3, 128, 8), (37, 256, 1)])
def test_router_matches_oracle(cuda_device, T, E, k):
    import torch

    from qk_b200.routing import routes

    rng = np.random.default_rng(T * 1000 + E)
    x = rng.normal(size=(T, 2048)).astype(np.float32)
    w = rng.normal(0, 0.02, (E, 2048)).astype(np.float32)
    active = np.ones(T, bool)
    active[::3] = False
    ids_o, w_o, probs_o = moe.routes(bf16_tensor(x, "cpu").float().numpy(), w, k, active)
    ids, weights, probs = routes(bf16_tensor(x, cuda_device), torch.from_numpy(w).to(cuda_device), k,
                                 torch.from_numpy(active).to(cuda_device), return_probs=True)
    ids = ids.cpu().numpy()
    _gap_ok(probs_o, ids, ids_o, k)
    same = (ids == ids_o).all(-1)
    assert same.mean() > 0.95
    got = to_f32(weights)
    ulp = np.abs(got.view(np.int32) - w_o.view(np.int32))
    assert ulp[same].max() <= 1
    assert (got[~active] == 0).all()
    np.testing.assert_allclose(probs.cpu().numpy(), probs_o, rtol=2e-5, atol=1e-9)


def test_router_ties_go_to_lower_index(cuda_device):
    import torch

    from qk_b200.routing import routes_from_logits

    logits = np.array([[1.0, 3.0, 3.0, 2.0, -1.0, 3.0], [0.0] * 6], np.float32)
    ids, weights = routes_from_logits(torch.from_numpy(logits).to(cuda_device), 3)
    np.testing.assert_array_equal(ids.cpu().numpy(), [[1, 2, 5], [0, 1, 2]])
    ids_o, w_o, _ = moe.routes(None, None, 3, logits=logits)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    np.testing.assert_array_equal(to_f32(weights), w_o)


@pytest.mark.parametrize("T,E,k", [(1, 512, 10), (8, 512, 10), (13, 64, 4), (64, 512, 10), (37, 256, 1)])
def test_two_launch_router_equals_the_one_launch_router(cuda_device, T, E, k):
    """router_logits (many CTAs) + routes_from_logits (a warp per token) give the ids, weights
    and probabilities of the one-launch cluster router bit for bit."""
    import torch

    from qk_b200.routing import router_logits, routes, routes_from_logits

    rng = np.random.default_rng(T * 7 + E)
    x = bf16_tensor(rng.normal(size=(T, 2048)).astype(np.float32), cuda_device)
    w = torch.from_numpy(rng.normal(0, 0.02, (E, 2048)).astype(np.float32)).to(cuda_device)
    active = torch.from_numpy(np.arange(T) % 5 != 2).to(cuda_device)
    ids1, w1, p1 = routes(x, w, k, active, return_probs=True)
    logits = router_logits(x, w)
    ids2, w2, p2 = routes_from_logits(logits, k, active, return_probs=True)
    assert torch.equal(ids1, ids2)
    assert torch.equal(w1.view(torch.int16), w2.view(torch.int16))
    assert torch.equal(p1.view(torch.int32), p2.view(torch.int32))
