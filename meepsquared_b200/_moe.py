"""LoRA on the experts of a mixture of experts, computed on the routed tokens only, on a B200.

The drop-in for ``meepsquared/_moe.py:_routed_forward`` (:70-126): the same function of the inputs, weights and
PEFT factors, with every step a libmeep2b kernel:

* ``route``      the permutation (:75-87): a stable counting sort of the flat expert ids on the device
                 (histogram, offset table, scatter), bit-exact with a stable sort, sentinels (ids >= E) last;
* ``gather``     selected = hidden[perm // k] and the routing weights in expert order;
* the gate/up projection with its adapters, SwiGLU applied in the product's epilogue (:118-119), which also keeps
  the pre-activation for the backward pass;
* the down projection with its adapters (:122);
* ``unpermute``  the weighted sum over each token's k rows (:123-126).

The backward pass mirrors it: the un-permute's gradient (and the routing weights'), the down projection's input
gradient with SwiGLU's backward in its epilogue, the gate/up projection's input gradient, the four adapter
reductions and the gather's gradient. The routing is computed once per layer call and its tile map shared by the
four grouped products.
"""

import os
from dataclasses import dataclass

import torch

from . import _grouped, _lib

_WEIGHT_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


@dataclass
class Routing:
    perm: torch.Tensor          # (S,) int64: flat assignment index of each row in expert order
    expert_ids_g: torch.Tensor  # (S,) int64: expert of each row, sentinels clamped to E-1
    offsets: torch.Tensor       # (E,) int32: end of each expert's rows
    inverse: torch.Tensor       # (S,) int64: row of each flat assignment
    weights_g: torch.Tensor     # (S,) routing weight of each row (the weights' dtype), or None
    num_tokens: int
    top_k: int
    num_experts: int
    tiles: tuple = None         # the tile map of the grouped products, built on first use

    def tile_map(self):
        if self.tiles is None:
            self.tiles = _grouped.TileMaps(self.offsets, self.perm.numel())
        return self.tiles


def route(top_k_index: torch.Tensor, top_k_weights, num_experts: int) -> Routing:
    """The routing permutation of _moe.py:75-87 for top_k_index (T, k); top_k_weights (T, k) may be None."""
    if not top_k_index.is_cuda:
        raise RuntimeError("route runs on a CUDA GPU")
    lib = _lib.load()
    tokens, k = top_k_index.shape
    ids = top_k_index.reshape(-1).to(torch.int64).contiguous()
    n = ids.numel()
    dev = ids.device
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    ids_g = torch.empty(n, dtype=torch.int64, device=dev)
    inverse = torch.empty(n, dtype=torch.int64, device=dev)
    offsets = torch.empty(num_experts, dtype=torch.int32, device=dev)
    ws_bytes = lib.meep2b_route_workspace_bytes(n, num_experts)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = _lib.stream_of(ids)
    _lib.check(lib.meep2b_route(_lib.ptr(ids), n, num_experts, _lib.ptr(perm), _lib.ptr(ids_g), _lib.ptr(offsets),
                                _lib.ptr(inverse), _lib.ptr(ws), ws_bytes, stream), "meep2b_route")
    weights_g = None
    if top_k_weights is not None:
        if top_k_weights.dtype not in _WEIGHT_DTYPES:
            raise TypeError(f"routing weights in {top_k_weights.dtype}: float32 or bf16 expected")
        weights_g = torch.empty(n, dtype=top_k_weights.dtype, device=dev)
    return Routing(perm, ids_g, offsets, inverse, weights_g, tokens, k, num_experts)


def route_logits(router_logits: torch.Tensor, top_k: int, num_experts: int, norm_topk_prob: bool = True,
                 probs: bool = True):
    """The router of Transformers' MoE blocks (Qwen3MoeTopKRouter.forward after its linear layer: softmax in float32,
    top-k, the weights renormalised when norm_topk_prob) and the routing permutation, in one pass over the logits.

    router_logits (T, E) float32 or bf16. Returns (probs (T, E) float32 or None, top_k_weights (T, k) float32,
    top_k_index (T, k) int64, Routing): the router's outputs, and the routing that routed_forward(..., routing=)
    takes instead of sorting the ids again."""
    if not router_logits.is_cuda:
        raise RuntimeError("route_logits runs on a CUDA GPU")
    if router_logits.dim() != 2 or router_logits.shape[1] != num_experts:
        raise ValueError(f"router logits {tuple(router_logits.shape)}: (tokens, {num_experts}) expected")
    if router_logits.dtype not in _WEIGHT_DTYPES:
        raise TypeError(f"router logits in {router_logits.dtype}: float32 or bf16 expected")
    lib = _lib.load()
    logits = router_logits.contiguous()
    tokens = logits.shape[0]
    n = tokens * top_k
    dev = logits.device
    p = torch.empty((tokens, num_experts), dtype=torch.float32, device=dev) if probs else None
    index = torch.empty((tokens, top_k), dtype=torch.int64, device=dev)
    weights = torch.empty((tokens, top_k), dtype=torch.float32, device=dev)
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    ids_g = torch.empty(n, dtype=torch.int64, device=dev)
    inverse = torch.empty(n, dtype=torch.int64, device=dev)
    offsets = torch.empty(num_experts, dtype=torch.int32, device=dev)
    ws_bytes = lib.meep2b_route_workspace_bytes(n, num_experts)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.check(lib.meep2b_route_logits(_lib.ptr(logits), _WEIGHT_DTYPES[logits.dtype], tokens, num_experts, top_k,
                                       int(bool(norm_topk_prob)), _lib.ptr(p), _lib.ptr(index), _lib.ptr(weights),
                                       _lib.ptr(perm), _lib.ptr(ids_g), _lib.ptr(offsets), _lib.ptr(inverse),
                                       _lib.ptr(ws), ws_bytes, _lib.stream_of(logits)), "meep2b_route_logits")
    routing = Routing(perm, ids_g, offsets, inverse, torch.empty(n, dtype=torch.float32, device=dev), tokens,
                      top_k, num_experts)
    return p, weights, index, routing


def gather(hidden: torch.Tensor, routing: Routing, top_k_weights=None) -> torch.Tensor:
    """selected = hidden[perm // k] with sentinel rows zeroed (_moe.py:80,87); fills routing.weights_g."""
    if hidden.dtype != torch.bfloat16:
        raise TypeError(f"the routed layer computes in bf16; hidden states are {hidden.dtype}")
    hidden = hidden.contiguous()
    rows = routing.perm.numel()
    sel = torch.empty((rows, hidden.shape[1]), dtype=hidden.dtype, device=hidden.device)
    w = top_k_weights.contiguous() if top_k_weights is not None else None
    wd = _WEIGHT_DTYPES[w.dtype] if w is not None else _lib.F32
    _lib.check(_lib.load().meep2b_gather(_lib.ptr(hidden), routing.num_tokens, hidden.shape[1], routing.top_k,
                                         _lib.ptr(routing.perm), _lib.ptr(routing.offsets), routing.num_experts,
                                         _lib.ptr(w), wd, _lib.ptr(routing.weights_g if w is not None else None),
                                         _lib.ptr(sel), _lib.stream_of(hidden)), "meep2b_gather")
    return sel


def unpermute(y: torch.Tensor, routing: Routing, weights_g=None) -> torch.Tensor:
    """(T, H) bf16: sum over each token's k rows of y[row] * weights_g[row] (unweighted when weights_g is None)."""
    y = y.contiguous()
    out = torch.empty((routing.num_tokens, y.shape[1]), dtype=torch.bfloat16, device=y.device)
    wd = _WEIGHT_DTYPES[weights_g.dtype] if weights_g is not None else _lib.F32
    _lib.check(_lib.load().meep2b_unpermute(_lib.ptr(y), _lib.ptr(routing.inverse), _lib.ptr(weights_g), wd,
                                            _lib.ptr(routing.offsets), routing.num_experts, routing.num_tokens,
                                            routing.top_k, y.shape[1], _lib.ptr(out), _lib.stream_of(y)),
               "meep2b_unpermute")
    return out


def combine(y_tok: torch.Tensor, routing: Routing, top_k_weights=None) -> torch.Tensor:
    """(T, H) bf16: the un-permute of rows stored token-major (row t * k + j: a product that placed its rows through
    the permutation, out_rows = perm): sum over j of y_tok[t * k + j] * top_k_weights[t, j] (unweighted when None),
    sentinel assignments contributing nothing. Each token's k rows are one contiguous read."""
    y_tok = y_tok.contiguous()
    out = torch.empty((routing.num_tokens, y_tok.shape[1]), dtype=torch.bfloat16, device=y_tok.device)
    w = top_k_weights.contiguous() if top_k_weights is not None else None
    wd = _WEIGHT_DTYPES[w.dtype] if w is not None else _lib.F32
    _lib.check(_lib.load().meep2b_combine(_lib.ptr(y_tok), _lib.ptr(routing.inverse), _lib.ptr(w), wd,
                                          _lib.ptr(routing.offsets), routing.num_experts, routing.num_tokens,
                                          routing.top_k, y_tok.shape[1], _lib.ptr(out), _lib.stream_of(y_tok)),
               "meep2b_combine")
    return out


def unpermute_backward(grad_out: torch.Tensor, y: torch.Tensor, routing: Routing):
    """(grad_y (S, H) bf16, grad_top_k_weights (T, k) float32) of unpermute with routing.weights_g."""
    grad_out = grad_out.contiguous()
    rows = routing.perm.numel()
    grad_y = torch.empty((rows, y.shape[1]), dtype=torch.bfloat16, device=y.device)
    grad_w = torch.empty(rows, dtype=torch.float32, device=y.device)
    w = routing.weights_g
    _lib.check(_lib.load().meep2b_unpermute_backward(_lib.ptr(grad_out), _lib.ptr(y), _lib.ptr(routing.perm),
                                                     _lib.ptr(w), _WEIGHT_DTYPES[w.dtype], _lib.ptr(routing.offsets),
                                                     routing.num_experts, rows, routing.top_k, y.shape[1],
                                                     _lib.ptr(grad_y), _lib.ptr(grad_w), _lib.stream_of(y)),
               "meep2b_unpermute_backward")
    return grad_y, grad_w.view(routing.num_tokens, routing.top_k)


@dataclass
class _Stacks:
    gate_up: torch.Tensor
    down: torch.Tensor
    gate_up_scale: torch.Tensor
    down_scale: torch.Tensor
    gate_up_bias: torch.Tensor
    down_bias: torch.Tensor
    is_transposed: bool
    num_experts: int
    scaling1: float
    scaling2: float


def _token_major_rows() -> bool:
    """MEEP2B_COMBINE=token: the down product (and the gate/up input gradient) store their rows token-major through
    the permutation for the streaming combine; the rows then go out by per-row stores. Default (sorted): rows in
    expert order, written as whole tiles by the epilogue's TMA stores, then the un-permute (measured faster on B200:
    the TMA-store epilogue gains more than the contiguous combine reads)."""
    return os.environ.get("MEEP2B_COMBINE", "sorted") == "token"


def routed_rows(routing: Routing, top_k_weights):
    """(token of each routed row (S,) int32, routing weight of each routed row (S,) float32): what the fused
    products read instead of gathered copies of the rows."""
    n = routing.perm.numel()
    dev = routing.perm.device
    token_rows = torch.empty(n, dtype=torch.int32, device=dev)
    w32 = torch.empty(n, dtype=torch.float32, device=dev)
    w = top_k_weights.contiguous() if top_k_weights is not None else None
    wd = _WEIGHT_DTYPES[w.dtype] if w is not None else _lib.F32
    _lib.check(_lib.load().meep2b_routed_rows(_lib.ptr(routing.perm), n, routing.top_k, _lib.ptr(w), wd,
                                              _lib.ptr(token_rows), _lib.ptr(w32 if w is not None else None),
                                              _lib.stream_of(routing.perm)), "meep2b_routed_rows")
    return token_rows, w32


class _RoutedExperts(torch.autograd.Function):
    """The whole routed layer: gradients for the hidden states, the routing weights and the four LoRA factors.

    MEEP2B_ROUTED_ROWS selects how the layer meets the routing (bf16 stacks without an expert bias; others always
    take "copy"):
      fold (default)  the forward gathers the hidden rows into expert order for the gate/up product; the backward
                      gathers the upstream gradient's rows (unweighted), and the down stack's input-gradient product
                      applies the routing weights and yields their gradient <dh, h> = <g, y> from its dSwiGLU
                      epilogue (the un-permute's backward, _moe.py:123-126, folded in: y is not kept); the adapter
                      reductions read the hidden and upstream-gradient rows where they are;
      gather          as fold, and the products read their x rows from the token-major tensors themselves (no
                      gathered copies; slower on B200: the rows arrive by cp.async, not TMA);
      copy            gathered copies, the un-permute's backward as its own kernel.
    """

    @staticmethod
    def forward(ctx, hidden, top_k_weights, lhs1, rhs1, lhs2, rhs2, top_k_index, st: _Stacks, routing=None):
        if routing is None:
            routing = route(top_k_index, top_k_weights, st.num_experts)
        elif routing.weights_g is None or routing.weights_g.dtype != top_k_weights.dtype:
            routing.weights_g = torch.empty(routing.perm.numel(), dtype=top_k_weights.dtype, device=hidden.device)
        mode = os.environ.get("MEEP2B_ROUTED_ROWS", "fold")
        if (isinstance(st.gate_up, _grouped.QuantStack) or isinstance(st.down, _grouped.QuantStack)
                or st.down_bias is not None or mode not in ("fold", "gather")):
            mode = "copy"
        tiles = routing.tile_map()
        t = st.is_transposed
        ad1 = _grouped._Adapters(lhs1.detach(), rhs1.detach(), t) if lhs1 is not None else None
        ad2 = _grouped._Adapters(lhs2.detach(), rhs2.detach(), t) if lhs2 is not None else None
        gate_up = _stack(st.gate_up)
        if isinstance(gate_up, _grouped.QuantStack):
            b_mn = 1 if t else 0
        else:
            _, b_mn = _grouped._stack_memory(gate_up, not t)
        if b_mn != 0:
            raise NotImplementedError("SwiGLU is fused for a gate/up stack stored (experts, 2I, hidden), k contiguous")
        two_i = gate_up.shape[2] if t else gate_up.shape[1]
        rows = routing.perm.numel()
        gu = torch.empty((rows, two_i), dtype=torch.bfloat16, device=hidden.device)
        token_rows = w32 = None
        if mode == "copy":
            x, x_rows, weights_g = gather(hidden, routing, top_k_weights), None, routing.weights_g
        else:
            token_rows, w32 = routed_rows(routing, top_k_weights)
            weights_g = w32
            if mode == "gather":
                x, x_rows = hidden, token_rows
            else:
                x, x_rows = gather(hidden, routing, None), None
        h, low1 = _grouped._launch(x, gate_up, st.gate_up_scale, routing.offsets, not t, ad1, st.scaling1,
                                   st.gate_up_bias, True, tiles=tiles, epilogue=_lib.EPI_SWIGLU, aux=gu,
                                   x_rows=x_rows)
        del gate_up  # a stack dequantised for this product alone is released before the next one is made
        if mode == "copy":
            y, low2 = _grouped._launch(h, _stack(st.down), st.down_scale, routing.offsets, not t, ad2, st.scaling2,
                                       st.down_bias, True, tiles=tiles)
            out = unpermute(y, routing, weights_g)
        elif _token_major_rows():
            # the combine of _moe.py:123-126 fused into the down product: its epilogue stores each row at the row's
            # flat assignment (token-major), and the weighted sum over a token's k rows reads one contiguous run
            y, low2 = _grouped._launch(h, _stack(st.down), st.down_scale, routing.offsets, not t, ad2, st.scaling2,
                                       st.down_bias, True, tiles=tiles, out_rows=routing.perm)
            out = combine(y, routing, top_k_weights)
            del y
        else:
            # rows in expert order (the epilogue's tiles go out whole by TMA stores), then the weighted un-permute
            y, low2 = _grouped._launch(h, _stack(st.down), st.down_scale, routing.offsets, not t, ad2, st.scaling2,
                                       st.down_bias, True, tiles=tiles)
            out = unpermute(y, routing, w32)
            del y
        kept = (x, gu, h, y) if mode == "copy" else (hidden, gu, h, token_rows, w32)
        ctx.save_for_backward(*kept, *(v for v in (low1, low2) if v is not None))
        ctx.routing, ctx.st, ctx.ad1, ctx.ad2, ctx.mode = routing, st, ad1, ad2, mode
        ctx.leaves = (lhs1, rhs1, lhs2, rhs2)  # the factors' own tensors: a gradient bucket may hold their slots
        ctx.has_low = (low1 is not None, low2 is not None)
        ctx.weights_dtype = top_k_weights.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        routing, st, ad1, ad2, mode = ctx.routing, ctx.st, ctx.ad1, ctx.ad2, ctx.mode
        saved = list(ctx.saved_tensors)
        if mode == "copy":
            sel, gu, h, y = saved[:4]
            lows = saved[4:]
        else:
            hidden, gu, h, token_rows, w32 = saved[:5]
            lows = saved[5:]
        low1 = lows.pop(0) if ctx.has_low[0] else None
        low2 = lows.pop(0) if ctx.has_low[1] else None
        tiles = routing.tile_map()
        t = st.is_transposed
        grad_out = grad_out.contiguous()
        if grad_out.dtype != torch.bfloat16:
            grad_out = grad_out.to(torch.bfloat16)
        if mode == "copy":
            grad_y, grad_w = unpermute_backward(grad_out, y, routing)
            dgu, low2b = _grouped._launch(grad_y, _stack(st.down), st.down_scale, routing.offsets, t, ad2,
                                          st.scaling2, None, True, backward=True, tiles=tiles,
                                          epilogue=_lib.EPI_DSWIGLU, aux=gu)
        else:
            # the down stack's input gradient over the upstream gradient's rows, each weighted by its routing weight,
            # SwiGLU's backward in the epilogue, and <dh, h> per row and 96 columns for the routing weights' gradient
            inter = gu.shape[1] // 2
            # every expert row's partials are written by the product; the sentinel rows' are not read
            parts = torch.empty((routing.perm.numel(), -(-inter // 96)), dtype=torch.float32, device=grad_out.device)
            if mode == "gather":
                g, g_rows = grad_out, token_rows
            else:
                g, g_rows = gather(grad_out, routing, None), None
            dgu, low2b = _grouped._launch(g, _stack(st.down), st.down_scale, routing.offsets, t, ad2, st.scaling2, None,
                                          True, backward=True, tiles=tiles, epilogue=_lib.EPI_DSWIGLU, aux=gu,
                                          x_rows=g_rows, row_scale=w32, w_grad=parts)
            grad_w = torch.empty(routing.perm.numel(), dtype=torch.float32, device=grad_out.device)
            _lib.check(_lib.load().meep2b_weight_grad(_lib.ptr(parts), parts.stride(0), parts.shape[1],
                                                      _lib.ptr(routing.perm), routing.perm.numel(),
                                                      _lib.ptr(routing.offsets), routing.num_experts, _lib.ptr(grad_w),
                                                      _lib.stream_of(parts)), "meep2b_weight_grad")
        grads = [None, None, None, None]
        if ad2 is not None:
            # the down projection's adapter gradients first: a data-parallel gradient bucket can start averaging
            # them while the gate/up input gradient runs
            first = dict(g=h, low=low2b)
            if mode == "copy":
                second = dict(g=grad_y, low=low2)
            else:
                second = dict(g=grad_out, low=low2, g_rows=token_rows, row_scale=w32)
            grads[2], grads[3] = _adapter_grads(ad2, ctx.leaves[2], ctx.leaves[3], first, second, routing.offsets,
                                                st.scaling2, tiles)
        gate_up_stack = _stack(st.gate_up)
        # quantised products store rows in order
        token_major = _token_major_rows() and not isinstance(gate_up_stack, _grouped.QuantStack)
        dsel, low1b = _grouped._launch(dgu, gate_up_stack, st.gate_up_scale, routing.offsets, t, ad1, st.scaling1,
                                       None, True, backward=True, tiles=tiles,
                                       out_rows=routing.perm if token_major else None)
        del gate_up_stack
        if ad1 is not None:
            if mode == "copy":
                first = dict(g=sel, low=low1b)
            else:
                first = dict(g=hidden, low=low1b, g_rows=token_rows)
            second = dict(g=dgu, low=low1)
            grads[0], grads[1] = _adapter_grads(ad1, ctx.leaves[0], ctx.leaves[1], first, second, routing.offsets,
                                                st.scaling1, tiles)
        grad_hidden = combine(dsel, routing, None) if token_major else unpermute(dsel, routing, None)
        grad_w = grad_w.view(routing.num_tokens, routing.top_k)
        return (grad_hidden, grad_w.to(ctx.weights_dtype), grads[0], grads[1], grads[2], grads[3], None, None, None)


def _adapter_grads(ad, lhs, rhs, first, second, offsets, scaling, tiles=None):
    """PEFT's (lhs, rhs) gradients of one stack's adapters from the two reductions of the backward pass (first: the
    factor the forward applies first, second: the other; _grouped.py:400-405), each written in its factor's own
    layout: (experts, n, 16) for lhs (E, out, r) or a transposed stack's lhs (E, in, r), (experts, 16, n) for rhs.
    At rank 16 a factor whose slot in a LoRA-gradient bucket is free (ddp.grad_slot) gets its gradient written
    there, and autograd adopts it without a copy."""
    from . import ddp

    rank = ad.rank
    lhs_first = ad.is_transposed  # a transposed stack applies lhs (E, in, r) first, else rhs^T
    spec = {"lhs": (first if lhs_first else second, 0, lhs), "rhs": (second if lhs_first else first, 1, rhs)}
    out = {}
    written = []
    for name, (red, layout, leaf) in spec.items():
        slot = ddp.grad_slot(leaf) if rank == RANK and leaf is not None else None
        if slot is not None and (slot.dtype != torch.bfloat16 or not slot.is_contiguous()):
            slot = None
        n = red["g"].shape[1]
        want = (offsets.numel(), n, RANK) if layout == 0 else (offsets.numel(), RANK, n)
        if slot is not None and tuple(slot.shape) != want:
            slot = None
        g = _grouped._reduce(red["g"], red["low"], offsets, scaling, g_rows=red.get("g_rows"),
                             row_scale=red.get("row_scale"), out=slot, layout=layout, tiles=tiles)
        out[name] = g if rank == RANK else (g[:, :, :rank] if layout == 0 else g[:, :rank, :])
        if slot is not None:
            written.append(leaf)
    for leaf in written:  # the bucket may start averaging these slots (they are complete in stream order)
        ddp.mark_written(leaf)
    return out["lhs"], out["rhs"]


RANK = _grouped.RANK_MULTIPLE


class _PerProduct:
    """A quantised stack dequantised to a bf16 copy each time a product reads it, the copy released after that
    product: for the forward product and again for the backward one, as the reference treats an FP8 stack
    (meepsquared/_fp8.py:140-156), so at most one layer stack is ever held in bf16."""

    def __init__(self, make):
        self.make = make


def _stack(s):
    return s.make() if isinstance(s, _PerProduct) else s


def _kernel_stack(experts, name):
    """(stack, scale) for the kernels. A bf16 stack as it is. A quantised one goes to the products as a QuantStack,
    dequantised in shared memory between the TMA load and the MMA: FP8 (e4m3) with its `<name>_scale_inv` (one
    scale per expert, applied in the epilogue, or a 128 x 128 grid of blocks) or NF4 (an NF4State in the
    attribute's place). A quantised stack without whole 64-weight blocks is dequantised to bf16 for each product
    instead, and so is every quantised stack with MEEP2B_DEQUANT=product (the dequantisation kernel's HBM traffic
    each time, the bf16 products' speed)."""
    from . import _fp8, _nf4

    weight = getattr(experts, name)
    per_product = os.environ.get("MEEP2B_DEQUANT", "fused") == "product"
    if isinstance(weight, _nf4.NF4State):
        fused = None if per_product else _grouped.QuantStack.from_nf4(weight)
        return (fused if fused is not None else _PerProduct(lambda: _nf4.dequantize(weight))), None
    if weight.dtype == torch.float8_e4m3fn:
        scale = getattr(experts, name + _fp8.STACK_SCALE)
        if _grouped.fp8_products(weight.device):
            # MEEPSQUARED_FP8_PRODUCTS=1: the products run on the FP8 tensor cores, the activations quantised per
            # row and 128-column tile (the reference's _moe passes products_fp8=None, so the switch decides)
            return _grouped.Fp8Stack.of(weight.detach(), scale), None
        # one scale per expert is applied to the accumulator, the codes converted exactly (_grouped.py:200-208);
        # a grid of block scales goes into the converted weights (quantize.py:131-157)
        per_expert = scale.dim() == 1
        epi_scale = scale.float().contiguous() if per_expert else None
        w8 = weight.detach()
        if per_expert:
            ones = torch.ones(w8.shape[0], device=w8.device, dtype=torch.float32)
            copy = _PerProduct(lambda: _fp8.dequantize_stack(w8, ones, torch.bfloat16))
        else:
            copy = _PerProduct(lambda: _fp8.dequantize_blocks(w8, scale))
        if per_product:
            return copy, epi_scale
        # the multipliers of a block-scaled stack are prepared once and kept while the stack and scale are unchanged
        cache = experts.__dict__.setdefault("_meep2b_quant_stacks", {})
        key = (weight.data_ptr(), weight._version, scale.data_ptr(), scale._version)
        hit = cache.get(name)
        if hit is not None and hit[0] == key:
            fused = hit[1]
        else:
            fused = _grouped.QuantStack.from_fp8(w8, scale)
            cache[name] = (key, fused)
        return (fused if fused is not None else copy), epi_scale
    if weight.dtype != torch.bfloat16:
        raise TypeError(f"expert stacks in bf16, FP8 (e4m3) or NF4; got {weight.dtype}")
    return weight.detach(), None


class _GatherRows(torch.autograd.Function):
    """The hidden rows in expert order (selected = hidden[perm // k], sentinel rows zero, _moe.py:80,87); the
    backward sums the rows' gradients back onto their tokens (the un-permute without weights)."""

    @staticmethod
    def forward(ctx, hidden, routing, top_k_weights):
        ctx.routing = routing
        return gather(hidden, routing, top_k_weights)

    @staticmethod
    def backward(ctx, grad):
        return unpermute(grad.contiguous().to(torch.bfloat16), ctx.routing, None), None, None


class _Combine(torch.autograd.Function):
    """out[t] = sum_j w[t, j] * y[row(t, j)] (_moe.py:123-126), sentinel rows contributing nothing; the backward
    gives the rows' gradients and the routing weights' gradient <g[t], y[row]>."""

    @staticmethod
    def forward(ctx, y, top_k_weights, routing):
        y = y.contiguous()
        ctx.save_for_backward(y)
        ctx.routing, ctx.weights_dtype = routing, top_k_weights.dtype
        return unpermute(y, routing, routing.weights_g)

    @staticmethod
    def backward(ctx, grad):
        (y,) = ctx.saved_tensors
        grad = grad.contiguous()
        if grad.dtype != torch.bfloat16:
            grad = grad.to(torch.bfloat16)
        grad_y, grad_w = unpermute_backward(grad, y, ctx.routing)
        return grad_y, grad_w.to(ctx.weights_dtype), None


def _default_swiglu(experts) -> bool:
    """Whether the module's gate is what the products' SwiGLU epilogues compute: Transformers' default gate
    (``_default_apply_gate``: the activation of the first half of the gate/up output times the second half) with a
    SiLU activation, on a gate/up stack stored (experts, 2I, hidden). A module without ``_apply_gate`` or ``act_fn``
    is taken as that default."""
    return not experts.is_transposed and _default_gate(experts)


def _default_gate(experts) -> bool:
    """Whether the module's gate is Transformers' default SwiGLU gate with a SiLU activation, whatever the layout of
    its stacks (the gate acts on the gate/up output, (rows, 2I) either way)."""
    if not experts.has_gate:
        return False
    gate = getattr(type(experts), "_apply_gate", None)
    if gate is not None:
        try:
            from transformers.integrations.moe import _default_apply_gate
        except ImportError:
            return False
        if gate is not _default_apply_gate:
            return False
    act = getattr(experts, "act_fn", None)
    return act is None or isinstance(act, torch.nn.SiLU) or type(act).__name__ == "SiLUActivation"


class _SwiGLU(torch.autograd.Function):
    """h = silu(gate) * up over the gate/up output (rows, 2I) on the library's kernel (meep2b_swiglu), the gate of
    the unfused layer when the module's gate is Transformers' default; the backward on meep2b_swiglu_backward."""

    @staticmethod
    def forward(ctx, gate_up):
        gate_up = gate_up.contiguous()
        rows, inter = gate_up.shape[0], gate_up.shape[1] // 2
        h = torch.empty((rows, inter), device=gate_up.device, dtype=torch.bfloat16)
        _lib.check(_lib.load().meep2b_swiglu(_lib.ptr(gate_up), rows, inter, _lib.ptr(h), _lib.stream_of(gate_up)),
                   "meep2b_swiglu")
        ctx.save_for_backward(gate_up)
        return h

    @staticmethod
    def backward(ctx, grad_h):
        (gate_up,) = ctx.saved_tensors
        grad_h = grad_h.contiguous().to(torch.bfloat16)
        rows, inter = gate_up.shape[0], gate_up.shape[1] // 2
        grad = torch.empty_like(gate_up)
        _lib.check(_lib.load().meep2b_swiglu_backward(_lib.ptr(gate_up), _lib.ptr(grad_h), rows, inter,
                                                      _lib.ptr(grad), _lib.stream_of(gate_up)),
                   "meep2b_swiglu_backward")
        return grad


def _routed_unfused(experts, hidden_states, top_k_index, top_k_weights, factors):
    """The routed layer for modules whose gate the epilogues do not compute (another activation or gating
    function, an ungated up projection, a transposed stack): the reference's structure (_moe.py:70-126) with every
    product on the grouped kernels (one autograd node per projection, as lora_linear), the routing, the gather and
    the weighted un-permute on this package's kernels, and the module's own gate or activation in between."""
    routing = route(top_k_index, top_k_weights, experts.num_experts)
    x = _GatherRows.apply(hidden_states.to(torch.bfloat16), routing, top_k_weights)
    t = bool(experts.is_transposed)

    def project(x, name, bias_name):
        stack, scale = _kernel_stack(experts, name)
        lhs, rhs, scaling = factors.get(name, (None, None, 1.0))
        cast = lambda f: f.to(torch.bfloat16) if f is not None and f.dtype != torch.bfloat16 else f  # noqa: E731
        bias = getattr(experts, bias_name) if experts.has_bias else None
        if bias is not None:
            bias = bias.detach().to(torch.bfloat16).contiguous()
        # The rows past the last expert's end (the sentinels, ids >= num_experts, which the reference masks,
        # _moe.py:113-115) are neither written by the products nor read by anything after them: the products'
        # tiles, the adapters' reductions and the combine cover the experts' rows only, and every operation in
        # between is row by row. So no pass over the whole output masks them.
        return _grouped._LoraGroupedProduct.apply(x.to(torch.bfloat16).contiguous(), _stack(stack), scale,
                                                  routing.offsets, t, cast(lhs), cast(rhs), float(scaling), bias, None)

    act = getattr(experts, "act_fn", None) or torch.nn.functional.silu
    if experts.has_gate:
        gate_up = project(x, "gate_up_proj", "gate_up_proj_bias")
        if _default_gate(experts) and gate_up.dtype == torch.bfloat16 and (gate_up.shape[1] // 2) % 8 == 0:
            h = _SwiGLU.apply(gate_up)
        elif hasattr(experts, "_apply_gate"):
            h = experts._apply_gate(gate_up)
        else:  # Transformers' default gate
            gate, up = gate_up.chunk(2, dim=-1)
            h = act(gate) * up
    else:
        h = act(project(x, "up_proj", "up_proj_bias"))
    y = project(h, "down_proj", "down_proj_bias")
    return _Combine.apply(y, top_k_weights, routing).to(hidden_states.dtype)


def _fp8_products_layer(experts, device) -> bool:
    """Whether the layer's products run on the FP8 tensor cores: an FP8 stack (a stack of another kind, an NF4State
    included, has no e4m3 dtype) and the reference's switch (fp8_products, _grouped.py:70-80)."""
    fp8 = any(getattr(getattr(experts, n, None), "dtype", None) == torch.float8_e4m3fn
              for n in ("gate_up_proj", "down_proj"))
    return fp8 and _grouped.fp8_products(device)


def routed_forward(experts, hidden_states, top_k_index, top_k_weights, factors, routing=None):
    """The routed layer of an experts module with its adapters: _moe._routed_forward's contract.

    experts: a Transformers experts module (num_experts, has_gate, has_bias, is_transposed, gate_up_proj or
    up_proj, down_proj; FP8 stacks with ``<name>_scale_inv`` of one scale per expert or a 128 x 128 block grid; NF4
    stacks as an ``_nf4.NF4State`` in the stack's place). factors: {stack name: (lhs, rhs, scaling)} in PEFT's
    layout. A gated module with Transformers' default SiLU gate and a gate/up stack stored (experts, 2I, hidden)
    runs the fused layer (SwiGLU in the products' epilogues, one autograd node); any other module runs the
    unfused form, its own gate or activation between the products. routing: the Routing of these ids from
    route_logits (the router fused with the sort), used instead of sorting them again by the fused layer.
    """
    if not hidden_states.is_cuda:
        raise RuntimeError("the routed layer runs on a CUDA GPU (compute capability 10.0)")
    large_rank = any(f[0] is not None and f[0].shape[2] > _grouped.RANK_MULTIPLE for f in factors.values())
    if not _default_swiglu(experts) or _fp8_products_layer(experts, hidden_states.device) or large_rank:
        # another gate, FP8 tensor-core products (their kernel has the plain epilogue), or adapters of rank above 16
        # (the products take them in 16-rank chunks)
        return _routed_unfused(experts, hidden_states, top_k_index, top_k_weights, factors)
    bias1 = experts.gate_up_proj_bias if experts.has_bias else None
    bias2 = experts.down_proj_bias if experts.has_bias else None
    lhs1, rhs1, s1 = factors.get("gate_up_proj", (None, None, 1.0))
    lhs2, rhs2, s2 = factors.get("down_proj", (None, None, 1.0))
    cast = lambda f: f.to(torch.bfloat16) if f is not None and f.dtype != torch.bfloat16 else f  # noqa: E731
    gate_up, scale1 = _kernel_stack(experts, "gate_up_proj")
    down, scale2 = _kernel_stack(experts, "down_proj")
    st = _Stacks(gate_up, down, scale1, scale2,
                 bias1.detach().to(torch.bfloat16).contiguous() if bias1 is not None else None,
                 bias2.detach().to(torch.bfloat16).contiguous() if bias2 is not None else None,
                 bool(experts.is_transposed), int(experts.num_experts), float(s1), float(s2))
    return _RoutedExperts.apply(hidden_states.to(torch.bfloat16), top_k_weights, cast(lhs1), cast(rhs1), cast(lhs2),
                                cast(rhs2), top_k_index, st, routing)
