"""The synthetic inputs the benchmarks use stand in for datasets that are not
available offline; they must be deterministic in their seed and have the
shapes and ranges the configurations name."""
import torch

from vggt_sparse.synthetic import clustered_layer, homography_views


def test_homography_views_are_seeded_and_in_range():
    a = homography_views(3, 56, seed=4)
    b = homography_views(3, 56, seed=4)
    c = homography_views(3, 56, seed=5)
    assert a.shape == (1, 3, 3, 56, 56)
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert float(a.min()) >= 0.0 and float(a.max()) <= 1.0
    # the views overlap (one texture) but differ (each has its own homography)
    assert 0.0 < float((a[0, 0] - a[0, 1]).abs().mean()) < 0.5


def test_clustered_layer_shapes_and_logit_scale():
    x = clustered_layer(2, centres=16, heads=4, seed=1)
    n = 2 * 1374
    assert x.q.shape == (4, n, 64) and x.kp.shape == (4, 2 * 1369, 64)
    assert x.ks.shape == (4, 10, 64) and x.vs.shape == (4, 10, 64)
    # random-pair logits q.k / sqrt(d) have a standard deviation near 3
    q, k = x.q.float(), x.kp.float()
    g = torch.Generator().manual_seed(0)
    i = torch.randint(0, q.shape[1], (2000,), generator=g)
    j = torch.randint(0, k.shape[1], (2000,), generator=g)
    logits = (q[:, i] * k[:, j]).sum(-1) / 8.0
    assert 2.0 < float(logits.std()) < 4.0
