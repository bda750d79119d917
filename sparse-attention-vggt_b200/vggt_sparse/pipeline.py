"""Running the layer on host (pinned) tensors with the transfers overlapped.

``HostPipeline(layer)`` takes each call's inputs in pinned host memory and
writes the output to a pinned host tensor.  ``layer`` is a SparseGlobalLayer
(estimator and attention run as two steps) or any layer called as
``layer(q, kp, vp, ks, vs, out=...)``, such as a FrameShardedLayer fed this
rank's shards.  Details for a SparseGlobalLayer: uploads run on one copy stream,
the download on another, the layer on the caller's current stream:

* q and the patch keys go up first, so the estimator starts while V and the
  specials are still in flight;
* two device buffer sets alternate between calls, so call i+1's uploads
  overlap call i's attention, and call i's download overlaps call i+1.

Every call still moves all of its inputs up and its output down; nothing is
cached between calls.  Calls return immediately; ``synchronize()`` (or an
event recorded on the current stream after ``wait_output``) orders host reads
of the outputs.
"""
import torch


class HostPipeline:
    def __init__(self, layer, depth=2):
        self.layer = layer
        self.depth = depth
        self._sets = [None] * depth
        self._free = [None] * depth     # event: set i's inputs and output may be reused
        self._out_ready = [None] * depth
        self._i = 0
        self._up = None
        self._down = None

    def _buffers(self, k, host):
        bufs = self._sets[k]
        if bufs is None or any(b.shape != h.shape or b.dtype != h.dtype for b, h in zip(bufs, host)):
            if self._free[k] is not None:
                # the old set may still be read by its call's compute or download
                self._free[k].synchronize()
            dev = torch.device("cuda", torch.cuda.current_device())
            bufs = [torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host]
            self._sets[k] = bufs
        return bufs

    def __call__(self, q, kp, vp, ks, vs, out, after=None):
        """q/kp/vp/ks/vs: pinned host tensors of one layer call; out: pinned
        host tensor of q's shape, written when the call's download ends.
        ``after``: an optional CUDA event the uploads wait for.  Returns the
        event that marks the end of the download."""
        if self._up is None:
            self._up = torch.cuda.Stream()
            self._down = torch.cuda.Stream()
        compute = torch.cuda.current_stream()
        k = self._i % self.depth
        self._i += 1
        host = (q, kp, vp, ks, vs)
        dq, dkp, dvp, dks, dvs, dout = self._buffers(k, host + (out,))
        up_qk, up_rest = torch.cuda.Event(), torch.cuda.Event()
        with torch.cuda.stream(self._up):
            if self._free[k] is not None:
                self._up.wait_event(self._free[k])
            if after is not None:
                self._up.wait_event(after)
            dq.copy_(q, non_blocking=True)
            dkp.copy_(kp, non_blocking=True)
            up_qk.record()
            dvp.copy_(vp, non_blocking=True)
            dks.copy_(ks, non_blocking=True)
            dvs.copy_(vs, non_blocking=True)
            up_rest.record()
        if hasattr(self.layer, "estimate"):
            compute.wait_event(up_qk)
            self.layer.estimate(dq, dkp, dks.shape[1])
            compute.wait_event(up_rest)
            self.layer.attend(dq, dkp, dvp, dks, dvs, out=dout)
        else:  # a layer that runs as one call (e.g. FrameShardedLayer)
            compute.wait_event(up_rest)
            self.layer(dq, dkp, dvp, dks, dvs, out=dout)
        done = torch.cuda.Event()
        done.record(compute)
        freed = torch.cuda.Event()
        with torch.cuda.stream(self._down):
            self._down.wait_event(done)
            out.copy_(dout, non_blocking=True)
            freed.record()
        self._free[k] = freed
        self._out_ready[k] = freed
        return freed

    def wait_output(self, stream=None):
        """Make ``stream`` (default: current) wait for every download issued."""
        stream = stream or torch.cuda.current_stream()
        for ev in self._out_ready:
            if ev is not None:
                stream.wait_event(ev)

    def synchronize(self):
        for ev in self._out_ready:
            if ev is not None:
                ev.synchronize()
