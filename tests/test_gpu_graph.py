"""The layer path (estimator, pairing, attention) has no host synchronisation,
so it can be captured in a CUDA graph and replayed on new inputs written in
place; replay output equals an eager run bit for bit."""
import pytest
import torch

import vggt_sparse
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,dense", [("topk", ()), ("mass", (0, 3))])
def test_layer_replays_from_a_cuda_graph(cuda, mode, dense):
    x = clustered_layer(4, centres=64, seed=11, device=cuda)
    y = clustered_layer(4, centres=64, seed=12, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode=mode, retention=0.25, tau=0.9,
                                          dense_heads=dense, kernel="tcgen05")
    ins = [t.clone() for t in (x.q, x.kp, x.vp, x.ks, x.vs)]
    out = torch.empty_like(x.q)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            layer(*ins, out=out)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer(*ins, out=out)
    for dst, src in zip(ins, (y.q, y.kp, y.vp, y.ks, y.vs)):
        dst.copy_(src)
    graph.replay()
    torch.cuda.synchronize()
    eager = vggt_sparse.SparseGlobalLayer(16, mode=mode, retention=0.25, tau=0.9,
                                          dense_heads=dense, kernel="tcgen05")
    want = eager(y.q, y.kp, y.vp, y.ks, y.vs)
    assert torch.equal(out, want)
