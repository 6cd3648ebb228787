"""Data-parallel host logic on CPU ranks (gloo, world size 2), the way the reference tests DDP
(tests/test_ddp.py there: gloo CPU processes): the flat LoRA-gradient bucket averages across ranks, autograd
accumulates into it in place, and a rank that fails before the exchange makes the other rank's collective end with
an error within the process group's timeout instead of hanging."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from meepsquared_b200.ddp import LoraGradBucket


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _average_worker(rank, world, port, queue):
    _init(rank, world, port)
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.zeros(3, 4, 2)), torch.nn.Parameter(torch.zeros(3, 2, 5))]
    bucket = LoraGradBucket(params)
    for step in range(2):
        bucket.zero()
        # each rank's loss differs; autograd accumulates into the bucket's views in place
        loss = (params[0] * (rank + 1)).sum() + (params[1] * (step + 1) * (rank + 2)).sum()
        loss.backward()
        bucket.reduce()
        queue.put((rank, step, params[0].grad.tolist(), params[1].grad.tolist(),
                   bucket.flat.data_ptr() == params[0].grad.data_ptr()))
    dist.barrier()
    dist.destroy_process_group()


class _WritesIntoSlots(torch.autograd.Function):
    """A layer that computes its factors' gradients straight into their bucket slots when they are free (as the
    routed layer's adapter reductions do), a fresh tensor otherwise."""

    @staticmethod
    def forward(ctx, x, a, b):
        ctx.save_for_backward(x)
        ctx.leaves = (a, b)
        return x * a.sum() + x * b.sum()

    @staticmethod
    def backward(ctx, g):
        from meepsquared_b200 import ddp

        (x,) = ctx.saved_tensors
        out = []
        for leaf in ctx.leaves:
            slot = ddp.grad_slot(leaf)
            dest = slot if slot is not None else torch.empty_like(leaf)
            dest.fill_(float((g * x).sum()))
            out.append(dest)
        return None, out[0], out[1]


def _release_worker(rank, world, port, queue):
    _init(rank, world, port)
    a, b = torch.nn.Parameter(torch.zeros(3, 4)), torch.nn.Parameter(torch.zeros(2, 5))
    bucket = LoraGradBucket([a, b])
    x = torch.full((6,), float(rank + 1))
    for step in range(2):
        bucket.release()
        _WritesIntoSlots.apply(x, a, b).sum().backward()
        adopted = a.grad.data_ptr() == bucket.flat.data_ptr() and b.grad.data_ptr() == bucket.flat[12:].data_ptr()
        bucket.reduce()
        queue.put((rank, step, adopted, a.grad.tolist(), b.grad.tolist(),
                   a.grad.data_ptr() == bucket.flat.data_ptr()))
    dist.barrier()
    dist.destroy_process_group()


class _WritesSegments(torch.autograd.Function):
    """A layer that writes its second factor's gradient first and reports each slot written (as the routed layer
    does for the down projection's adapters before the gate/up projection's)."""

    @staticmethod
    def forward(ctx, x, a, b):
        ctx.save_for_backward(x)
        ctx.leaves = (a, b)
        return x * a.sum() + x * b.sum()

    @staticmethod
    def backward(ctx, g):
        from meepsquared_b200 import ddp

        (x,) = ctx.saved_tensors
        a, b = ctx.leaves
        sb = ddp.grad_slot(b)
        sb.fill_(float((g * x).sum()) * 2)
        ddp.mark_written(b)  # completes the first segment: its average starts now
        started = list(ctx.bucket._started)
        sa = ddp.grad_slot(a)
        sa.fill_(float((g * x).sum()))
        ddp.mark_written(a)
        ctx.bucket.seen.append((started, list(ctx.bucket._started)))
        return None, sa, sb


def _segments_worker(rank, world, port, queue):
    _init(rank, world, port)
    a, b = torch.nn.Parameter(torch.zeros(3, 4)), torch.nn.Parameter(torch.zeros(2, 5))
    bucket = LoraGradBucket([a, b], segments=[[b], [a]])
    bucket.seen = []
    x = torch.full((6,), float(rank + 1))
    for step in range(2):
        bucket.release()
        y = _WritesSegments.apply(x, a, b)
        y.grad_fn.bucket = bucket
        y.sum().backward()
        bucket.reduce()
        queue.put((rank, step, bucket.seen[-1], a.grad.tolist(), b.grad.tolist(),
                   b.grad.data_ptr() == bucket.flat.data_ptr(), a.grad.data_ptr() == bucket.flat[10:].data_ptr()))
    dist.barrier()
    dist.destroy_process_group()


def _failing_worker(rank, world, port, queue):
    _init(rank, world, port, timeout_s=5)
    params = [torch.nn.Parameter(torch.zeros(8))]
    bucket = LoraGradBucket(params)
    if rank == 1:
        queue.put((rank, "left"))
        queue.close()
        queue.join_thread()  # the message is out before the process goes
        os._exit(3)  # leaves between steps, before the exchange: no collective of its own in flight
    params[0].sum().backward()
    try:
        bucket.reduce()
        queue.put((rank, "returned"))
    except Exception as exc:  # the collective ends with an error (timeout or closed connection)
        queue.put((rank, f"error: {type(exc).__name__}"))
    queue.close()
    queue.join_thread()
    os._exit(0)


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    items = []
    expected = {"_average_worker": 2 * world, "_release_worker": 2 * world, "_segments_worker": 2 * world,
                "_failing_worker": world}[fn.__name__]
    import queue as _queue
    try:
        while len(items) < expected:
            items.append(queue.get(timeout=120))
    except _queue.Empty:
        pass
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    return procs, items


def test_the_bucket_averages_lora_gradients_across_ranks():
    procs, items = _run(_average_worker)
    assert all(p.exitcode == 0 for p in procs)
    assert len(items) == 4
    for rank, step, g0, g1, shares_storage in items:
        assert shares_storage
        g0, g1 = torch.tensor(g0), torch.tensor(g1)
        torch.testing.assert_close(g0, torch.full_like(g0, (1 + 2) / 2))
        torch.testing.assert_close(g1, torch.full_like(g1, (step + 1) * (2 + 3) / 2))


def test_a_rank_that_leaves_before_the_exchange_ends_the_other_ranks_collective_with_an_error():
    procs, items = _run(_failing_worker)
    outcome = dict(items)
    assert outcome[1] == "left"
    assert outcome[0].startswith("error"), outcome[0]
    assert procs[0].exitcode == 0


def test_gradients_written_into_the_bucket_are_adopted_without_copies_and_averaged():
    """release() then backward: the layer writes each gradient into the parameter's slot of the flat buffer and
    autograd adopts it as .grad (no zeroing, no add); reduce() averages the buffer across the ranks."""
    procs, items = _run(_release_worker)
    assert all(p.exitcode == 0 for p in procs)
    assert len(items) == 4
    for rank, step, adopted, ga, gb, in_bucket in items:
        assert adopted and in_bucket
        # each rank's gradient is 6 (rank + 1): the average over ranks 0 and 1 is 9
        torch.testing.assert_close(torch.tensor(ga), torch.full((3, 4), 9.0))
        torch.testing.assert_close(torch.tensor(gb), torch.full((2, 5), 9.0))


def test_a_gradient_that_arrives_elsewhere_is_copied_into_the_bucket():
    """A parameter whose gradient autograd accumulated on its own (the slot was taken: .grad already set) or that
    got none: adopt() leaves every .grad a view of the flat buffer with the right values."""
    a, b, c = (torch.nn.Parameter(torch.zeros(4)) for _ in range(3))
    bucket = LoraGradBucket([a, b, c])
    bucket.release()
    a.grad = torch.full((4,), 2.0)        # set outside the bucket
    (b * 3.0).sum().backward()             # autograd's own accumulation into a fresh tensor
    bucket.adopt()
    assert a.grad.data_ptr() == bucket.flat.data_ptr()
    assert b.grad.data_ptr() == bucket.flat[4:].data_ptr() and c.grad.data_ptr() == bucket.flat[8:].data_ptr()
    torch.testing.assert_close(bucket.flat, torch.tensor([2.0] * 4 + [3.0] * 4 + [0.0] * 4))
    # with the slots free, a second layer call would write into them; with .grad set they are not offered
    from meepsquared_b200 import ddp

    assert ddp.grad_slot(a) is None
    bucket.release()
    assert ddp.grad_slot(a) is not None and ddp.grad_slot(a).data_ptr() == bucket.flat.data_ptr()


def test_a_segment_starts_averaging_as_soon_as_its_gradients_are_written():
    """segments=[[b], [a]]: the layer writes b's slot first; b's average starts then (before a is written), a's
    when a is written; reduce() joins both. The buffer holds the segments in that order and both gradients are the
    averages over the ranks."""
    procs, items = _run(_segments_worker)
    assert all(p.exitcode == 0 for p in procs)
    assert len(items) == 4
    for rank, step, (after_b, after_a), ga, gb, b_first, a_after in items:
        assert after_b == [True, False] and after_a == [True, True]
        assert b_first and a_after
        torch.testing.assert_close(torch.tensor(ga), torch.full((3, 4), 9.0))
        torch.testing.assert_close(torch.tensor(gb), torch.full((2, 5), 18.0))


def test_segments_must_partition_the_parameters():
    a, b = torch.nn.Parameter(torch.zeros(2)), torch.nn.Parameter(torch.zeros(3))
    with pytest.raises(ValueError):
        LoraGradBucket([a, b], segments=[[a]])
    with pytest.raises(ValueError):
        LoraGradBucket([a, b], segments=[[a, b], [b]])


def test_a_written_gradient_replaced_by_a_hook_is_refused():
    """With segments a slot may be averaging already when autograd stores the gradient: a hook that replaces the
    written gradient would race with it, so adopt() refuses instead of copying."""
    from meepsquared_b200 import ddp

    a = torch.nn.Parameter(torch.zeros(4))
    bucket = LoraGradBucket([a], segments=[[a]])
    bucket.release()
    slot = ddp.grad_slot(a)
    slot.fill_(1.0)
    ddp.mark_written(a)
    a.grad = torch.full((4,), 2.0)  # what a replacing hook would leave
    with pytest.raises(RuntimeError):
        bucket.adopt()
