"""Data parallelism of the expert layer, as the reference's DDP partitions it: every rank routes and computes its
own token batch with full replicas of the frozen stacks and of the LoRA factors, and the only exchange is the
average of the LoRA factors' gradients (torch DDP's bucketed all-reduce under HF Trainer in the reference,
meepsquared/_trl.py:240-244, benchmarks/multi_gpu.py:53-61).

Here the gradients of all adapters live in ONE flat buffer (each factor's ``.grad`` is a view into it, so autograd
accumulates in place) and one NCCL all-reduce (ReduceOp.AVG) averages it: one launch per step, sized for
NVLink / NVSwitch rather than for buckets. ``reduce_async`` issues it on a side stream so that it can overlap the
remaining backward work of the step.
"""

import torch
import torch.distributed as dist


class LoraGradBucket:
    """One contiguous gradient buffer for the given parameters, all-reduced (averaged) across the process group."""

    def __init__(self, params, group=None):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dtypes = {p.dtype for p in self.params}
        if len(dtypes) != 1:
            raise ValueError(f"one dtype per bucket, got {dtypes}")
        device = self.params[0].device
        total = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(total, dtype=self.params[0].dtype, device=device)
        self.group = group
        off = 0
        for p in self.params:
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()
        self._work = None
        self._stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def zero(self):
        self.flat.zero_()

    def _world(self):
        return dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1

    def reduce(self):
        """Averages the gradients over the ranks (blocking on the current stream's order)."""
        if self._world() > 1:
            if self.flat.is_cuda:
                dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group)
            else:  # gloo has no AVG
                dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
                self.flat.div_(self._world())
        return self.flat

    def reduce_async(self):
        """Starts the average on a side stream that waits for the gradients; wait() joins it."""
        if self._world() <= 1:
            return
        if self._stream is None:
            self.reduce()
            return
        self._stream.wait_stream(torch.cuda.current_stream(self.flat.device))
        with torch.cuda.stream(self._stream):
            self._work = dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group, async_op=True)

    def wait(self):
        if self._work is not None:
            self._work.wait()
            torch.cuda.current_stream(self.flat.device).wait_stream(self._stream)
            self._work = None
