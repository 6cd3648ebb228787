"""Data parallelism of the expert layer, as the reference's DDP partitions it: every rank routes and computes its
own token batch with full replicas of the frozen stacks and of the LoRA factors, and the only exchange is the
average of the LoRA factors' gradients (torch DDP's bucketed all-reduce under HF Trainer in the reference,
meepsquared/_trl.py:240-244, benchmarks/multi_gpu.py:53-61).

Here the gradients of all adapters live in ONE flat buffer (each factor's ``.grad`` is a view into it; the routed
layer writes its adapter gradients straight into those views) and NCCL all-reduces (ReduceOp.AVG) average it, one
per segment of the buffer: with the down projection's adapters in one segment and the gate/up projection's in
another, the first average starts on a side stream as soon as the layer has written those gradients, beside the
rest of the backward pass (the gate/up input gradient), and the second at the end of the step. Sized for NVLink /
NVSwitch: two launches per step, not many small buckets.
"""

import torch
import torch.distributed as dist
from torch.utils.weak import WeakIdKeyDictionary

# parameter -> its view of a bucket's flat buffer (keyed by identity: tensors do not compare by ==)
_SLOTS = WeakIdKeyDictionary()
# parameter -> the bucket that holds its slot
_OWNER = WeakIdKeyDictionary()


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
    first make every parameter's `.grad` its view again, whichever way the gradients arrived.

    segments: the parameters grouped in the order their gradients become ready in the backward pass (the routed
    layer finishes the down projection's adapters before the gate/up projection's). Each segment is a contiguous
    slice of the buffer; when a layer has written every gradient of a segment into its slots (mark_written), that
    slice's average starts at once on a side stream, beside the rest of the backward pass, and reduce() averages
    whatever has not started yet and joins the rest. Every rank writes the segments in the same order, so the
    collectives match. A gradient written into a slot must then reach `.grad` as it is: a gradient hook that
    replaces it is refused (adopt raises). Default: one segment, averaged by reduce()."""

    def __init__(self, params, group=None, segments=None):
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("no trainable parameters")
        if segments is None:
            segments = [params]
        segments = [[p for p in seg if p.requires_grad] for seg in segments]
        segments = [seg for seg in segments if seg]
        flat_order = [p for seg in segments for p in seg]
        if {id(p) for p in flat_order} != {id(p) for p in params} or len(flat_order) != len(params):
            raise ValueError("segments must hold every trainable parameter exactly once")
        self.params = flat_order
        dtypes = {p.dtype for p in self.params}
        if len(dtypes) != 1:
            raise ValueError(f"one dtype per bucket, got {dtypes}")
        device = self.params[0].device
        total = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(total, dtype=self.params[0].dtype, device=device)
        self.group = group
        self.views = []
        self.segments = []  # (first, end) element range of each segment in the flat buffer, and its parameters
        off = 0
        for seg in segments:
            first = off
            for p in seg:
                view = self.flat[off:off + p.numel()].view_as(p)
                p.grad = view
                _SLOTS[p] = view
                _OWNER[p] = self
                self.views.append(view)
                off += p.numel()
            self.segments.append((first, off, [id(p) for p in seg]))
        self._written = set()
        self._started = [False] * len(self.segments)
        self._works = []  # (work, segment index) of the averages in flight
        self._stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def zero(self):
        self.flat.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v
        self._new_step()

    def release(self):
        """Clears every parameter's `.grad` (nothing is zeroed): the next backward writes or adopts fresh gradients."""
        for p in self.params:
            p.grad = None
        self._new_step()

    def _new_step(self):
        if self._works:
            self.wait()
        self._written.clear()
        self._started = [False] * len(self.segments)

    def adopt(self):
        """Makes each parameter's `.grad` its view of the buffer: a gradient autograd adopted from the layer is
        there already; another one is copied in; a parameter that got none has its view zeroed."""
        for p, v in zip(self.params, self.views):
            g = p.grad
            moved = g is not None and (g.data_ptr() != v.data_ptr() or g.stride() != v.stride())
            if id(p) in self._written and moved:
                # the slot's segment may be averaging already: a copy now would race with it
                raise RuntimeError("a gradient written into its bucket slot was not adopted as it is (a gradient "
                                   "hook on a LoRA parameter?): build the bucket without segments")
            if g is None:
                if id(p) not in self._written:
                    v.zero_()
            elif moved:
                v.copy_(g)
            p.grad = v

    def _world(self):
        return dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1

    def _start(self, i):
        """Starts the average of segment i (its gradients are in the buffer, in the current stream's order)."""
        self._started[i] = True
        if self._world() <= 1:
            return
        first, end, _ = self.segments[i]
        part = self.flat[first:end]
        if self._stream is None:  # gloo has no AVG: sum now, divide when joined
            self._works.append((dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group, async_op=True), i))
            return
        self._stream.wait_stream(torch.cuda.current_stream(self.flat.device))
        with torch.cuda.stream(self._stream):
            work = dist.all_reduce(part, op=dist.ReduceOp.AVG, group=self.group, async_op=True)
        self._works.append((work, i))

    def mark_written(self, param):
        """A layer wrote param's gradient into its slot (on the current stream); when that completes a segment,
        the segment's average starts."""
        self._written.add(id(param))
        for i, (_, _, ids) in enumerate(self.segments):
            if not self._started[i] and id(param) in ids and all(j in self._written for j in ids):
                self._start(i)

    def reduce(self):
        """Averages the gradients over the ranks: the segments not started yet now, in order, then joins every
        average (the current stream waits for them)."""
        self.adopt()
        for i in range(len(self.segments)):
            if not self._started[i]:
                self._start(i)
        self.wait()
        return self.flat

    def reduce_async(self):
        """Starts the average of every segment not started yet on the side stream; wait() joins them."""
        self.adopt()
        for i in range(len(self.segments)):
            if not self._started[i]:
                self._start(i)

    def wait(self):
        for work, i in self._works:
            work.wait()
            if self._stream is None:
                first, end, _ = self.segments[i]
                self.flat[first:end].div_(self._world())
        if self._works and self._stream is not None:
            torch.cuda.current_stream(self.flat.device).wait_stream(self._stream)
        self._works = []


def mark_written(param):
    """Called by a layer that wrote param's gradient straight into its bucket slot (grad_slot): lets the bucket
    start averaging the slot's segment as soon as the segment is complete."""
    bucket = _OWNER.get(param)
    if bucket is not None:
        bucket.mark_written(param)
