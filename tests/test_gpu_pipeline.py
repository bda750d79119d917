"""HostPipeline runs a stream of layer calls on pinned host tensors with the
copies of neighbouring calls overlapped; each call's host output equals the
same layer run on device copies of its inputs, bit for bit, and the outputs
of calls that share a host buffer come out in order."""
import pytest
import torch

import vggt_sparse
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,dense", [("topk", ()), ("mass", (2,))])
def test_pipeline_matches_device_calls(cuda, mode, dense):
    layers = [clustered_layer(4, centres=64, seed=20 + i, device=cuda) for i in range(5)]
    layer = vggt_sparse.SparseGlobalLayer(16, mode=mode, retention=0.25, tau=0.9,
                                          dense_heads=dense, kernel="tcgen05")
    want = [layer(x.q, x.kp, x.vp, x.ks, x.vs).cpu() for x in layers]
    host = [[t.cpu().pin_memory() for t in (x.q, x.kp, x.vp, x.ks, x.vs)] for x in layers]
    outs = [torch.empty(x.q.shape, dtype=x.q.dtype).pin_memory() for x in layers]
    pipe = vggt_sparse.HostPipeline(layer)
    for h, o in zip(host, outs):
        pipe(*h, out=o)
    pipe.synchronize()
    for got, ref in zip(outs, want):
        assert torch.equal(got, ref)


def test_pipeline_reuses_one_output_buffer_in_order(cuda):
    layers = [clustered_layer(2, centres=32, seed=40 + i, device=cuda) for i in range(3)]
    layer = vggt_sparse.SparseGlobalLayer(16, mode="topk", retention=0.25, kernel="tcgen05")
    host = [[t.cpu().pin_memory() for t in (x.q, x.kp, x.vp, x.ks, x.vs)] for x in layers]
    out = torch.empty(layers[0].q.shape, dtype=layers[0].q.dtype).pin_memory()
    pipe = vggt_sparse.HostPipeline(layer)
    for h in host:
        pipe(*h, out=out)
    pipe.synchronize()
    last = layers[-1]
    assert torch.equal(out, layer(last.q, last.kp, last.vp, last.ks, last.vs).cpu())


def test_pipeline_follows_a_change_of_shape(cuda):
    small = clustered_layer(2, centres=32, seed=50, device=cuda)
    big = clustered_layer(4, centres=32, seed=51, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode="topk", retention=0.25, kernel="tcgen05")
    pipe = vggt_sparse.HostPipeline(layer)
    outs = []
    for x in (small, big, small, big):
        h = [t.cpu().pin_memory() for t in (x.q, x.kp, x.vp, x.ks, x.vs)]
        o = torch.empty(x.q.shape, dtype=x.q.dtype).pin_memory()
        pipe(*h, out=o)
        outs.append((x, o))
    pipe.synchronize()
    for x, o in outs:
        assert torch.equal(o, layer(x.q, x.kp, x.vp, x.ks, x.vs).cpu())
