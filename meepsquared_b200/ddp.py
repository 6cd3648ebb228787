"""Data parallelism of the expert layer, as the reference's DDP partitions it: every rank routes and computes its
own token batch with full replicas of the frozen stacks and of the LoRA factors, and the only exchange is the
average of the LoRA factors' gradients (torch DDP's bucketed all-reduce under HF Trainer in the reference,
meepsquared/_trl.py:240-244, benchmarks/multi_gpu.py:53-61).

Here the gradients of all adapters live in ONE flat buffer (each factor's ``.grad`` is a view into it; the routed
layer writes its adapter gradients straight into those views) and one NCCL all-reduce (ReduceOp.AVG) averages it:
one launch per step, sized for NVLink / NVSwitch rather than for buckets. ``reduce_async`` issues it on a side
stream so that it can overlap the remaining backward work of the step.
"""

import torch
import torch.distributed as dist
from torch.utils.weak import WeakIdKeyDictionary

# parameter -> its view of a bucket's flat buffer (keyed by identity: tensors do not compare by ==)
_SLOTS = WeakIdKeyDictionary()


def grad_slot(param):
    """The view of a LoRA-gradient bucket that `param`'s gradient is to be written into, when `param` belongs to a
    bucket and holds no gradient yet (LoraGradBucket.release()); None otherwise. A backward pass that computes the
    gradient straight into this view and returns it lets autograd adopt it as `.grad` without a copy or an add."""
    view = _SLOTS.get(param)
    if view is None or param.grad is not None:
        return None
    return view.view_as(view)  # a new alias of the slot: autograd adopts a gradient only if nothing else holds it


class LoraGradBucket:
    """One contiguous gradient buffer for the given parameters, all-reduced (averaged) across the process group.

    Two ways to fill it each step: zero() then backward (autograd adds each gradient into the parameter's view), or
    release() then backward, where a layer that knows the bucket (the routed layer's adapter reductions, through
    grad_slot) writes each gradient into its view directly and nothing is zeroed or added. reduce() / reduce_async()
    first make every parameter's `.grad` its view again, whichever way the gradients arrived."""

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
        self.views = []
        off = 0
        for p in self.params:
            view = self.flat[off:off + p.numel()].view_as(p)
            p.grad = view
            _SLOTS[p] = view
            self.views.append(view)
            off += p.numel()
        self._work = None
        self._stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def zero(self):
        self.flat.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v

    def release(self):
        """Clears every parameter's `.grad` (nothing is zeroed): the next backward writes or adopts fresh gradients."""
        for p in self.params:
            p.grad = None

    def adopt(self):
        """Makes each parameter's `.grad` its view of the buffer: a gradient autograd adopted from the layer is
        there already; another one is copied in; a parameter that got none has its view zeroed."""
        for p, v in zip(self.params, self.views):
            g = p.grad
            if g is None:
                v.zero_()
            elif g.data_ptr() != v.data_ptr() or g.stride() != v.stride():
                v.copy_(g)
            p.grad = v

    def _world(self):
        return dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1

    def reduce(self):
        """Averages the gradients over the ranks (blocking on the current stream's order)."""
        self.adopt()
        if self._world() > 1:
            if self.flat.is_cuda:
                dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group)
            else:  # gloo has no AVG
                dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
                self.flat.div_(self._world())
        return self.flat

    def reduce_async(self):
        """Starts the average on a side stream that waits for the gradients; wait() joins it."""
        self.adopt()
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
