"""Host-resident batches through mosaic_attn_func with the PCIe copies overlapped.

The reference's attention is called on tensors already on the GPU. A caller whose
fields live in host memory (an inference service, an ensemble driver that stages
members from the host) pays a host->device copy of q, k, v and the gates and a
device->host copy of the output per call; done in order on one stream, those
copies take several times longer than the attention itself. `StreamedAttention`
runs batch i's attention while batch i+1 is copied in and batch i-1 is copied
out, on three CUDA streams, with `depth` device buffer sets so that no copy
overwrites a buffer that a kernel still reads:

    pipe = StreamedAttention(device, 1024, 64, 24)
    for i, (q, k, v, w) in enumerate(host_batches):   # pinned host tensors
        pipe.submit(q, k, v, w, out_host[i])
    pipe.join()     # the caller's stream now waits for every copy-out

Results equal calling `mosaic_attn_func` on each batch in order.
"""
import torch

from .primitives import mosaic_attn_func

__all__ = ["StreamedAttention"]


class StreamedAttention:
    def __init__(self, device, block_attn_size, sparse_block_size, sparse_block_count, block_attn_only=False,
                 no_compression=False, depth=2):
        if depth < 2:
            raise ValueError("depth must be >= 2 (one buffer set computes while the next one fills)")
        self.device = torch.device(device)
        self.args = (block_attn_size, sparse_block_size, sparse_block_count, block_attn_only, no_compression)
        self.depth = depth
        self.s_in = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self.slots = [None] * depth  # device buffers per slot
        self.e_in = [torch.cuda.Event() for _ in range(depth)]
        self.e_comp = [torch.cuda.Event() for _ in range(depth)]
        self.e_out = [torch.cuda.Event() for _ in range(depth)]
        self.used = [False] * depth
        self.count = 0
        self._started = False

    def _buffers(self, j, host):
        cur = self.slots[j]
        if cur is None or any(cur[n].shape != t.shape or cur[n].dtype != t.dtype for n, t in host.items()):
            cur = {n: torch.empty(t.shape, dtype=t.dtype, device=self.device) for n, t in host.items()}
            self.slots[j] = cur
        return cur

    def submit(self, q, k, v, weight_ba_cmp_slc, out):
        """Queues one batch: host q, k, v, gates (pinned, for truly asynchronous
        copies) in, attention, output into the host tensor `out` (pinned)."""
        if not self._started:
            # everything the caller queued before (e.g. a start event) comes first
            base = torch.cuda.current_stream(self.device)
            for s in (self.s_in, self.s_comp, self.s_out):
                s.wait_stream(base)
            self._started = True
        j = self.count % self.depth
        host = {"q": q, "k": k, "v": v, "w": weight_ba_cmp_slc}
        dev = self._buffers(j, host)
        if self.used[j]:
            self.s_in.wait_event(self.e_comp[j])  # the attention that read this slot is done
        with torch.cuda.stream(self.s_in):
            for n, t in host.items():
                dev[n].copy_(t, non_blocking=True)
            self.e_in[j].record(self.s_in)
        self.s_comp.wait_event(self.e_in[j])
        with torch.cuda.stream(self.s_comp):
            o = mosaic_attn_func(dev["q"], dev["k"], dev["v"], dev["w"], *self.args)
            self.e_comp[j].record(self.s_comp)
        self.s_out.wait_event(self.e_comp[j])
        with torch.cuda.stream(self.s_out):
            out.copy_(o, non_blocking=True)
            o.record_stream(self.s_out)  # the allocator may reuse o only after the copy
            self.e_out[j].record(self.s_out)
        self.used[j] = True
        self.count += 1

    def join(self):
        """Makes the caller's current stream wait for every queued batch."""
        base = torch.cuda.current_stream(self.device)
        for s in (self.s_in, self.s_comp, self.s_out):
            base.wait_stream(s)
        self._started = False
