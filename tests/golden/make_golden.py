"""Writes the golden vectors of tests/golden/ by running the REFERENCE's own code (thinkube/meepsquared) on CPU.

    python tests/golden/make_golden.py /path/to/meepsquared/checkout

Run once in a container that holds the reference; the .npz files it writes are committed, and the tests read only
those (the reference does not exist where the GPU tests run). It imports the reference's modules through a stub
package (its __init__ pulls in trl, which the path does not need), and the vendored axolotl ``quantize`` module
with a stand-in for bitsandbytes (only its FP8 functions, which are pure PyTorch, are called). Everything is
seeded; bf16 tensors are stored as uint16 bit patterns, e4m3 as uint8 codes.

Files:
  tile_map.npz      reference _grouped.tile_map on the reference tests' cases and seeded random offsets
  routing.npz       the reference's sort / histc / cumsum on seeded router outputs (torch.sort, stable and not)
  layer_small.npz   _moe._routed_forward, forward and backward, float32, SMALL config (and a sentinel case)
  layer_config1.npz the same at BASELINE config 1 (T=512, H=256, I=512, E=8, top-2, r=8): slices and norms
  layer_bf16.npz    _moe._routed_forward on a bf16 model (config 2's H, I and rank, 128 tokens, 16 experts;
                    the adapters' gradients of every fifth expert)
  fp8_stack.npz     _fp8.quantize_stack / dequantize_stack (one scale per expert)
  fp8_block.npz     axolotl quantize.quantize_fp8 / dequantize_fp8 with 128x128 block scales, tails included
  grouped.npz       _grouped.reference_lora forward + backward, float32, the reference tests' ragged case
"""

import importlib
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import layer_inputs  # noqa: E402


# The bf16 case: config 2's hidden and intermediate sizes and rank, 128 tokens over 16 experts
LAYER_BF16 = dict(layer_inputs.QWEN3_30B, tokens=128, experts=16)


def import_reference(root):
    pkg = types.ModuleType("meepsquared")
    pkg.__path__ = [os.path.join(root, "src", "meepsquared")]
    sys.modules["meepsquared"] = pkg
    return (importlib.import_module("meepsquared._moe"), importlib.import_module("meepsquared._grouped"),
            importlib.import_module("meepsquared._fp8"))


def import_quantize(root):
    """The vendored axolotl quantize module, bitsandbytes replaced by a stand-in (its ctypes paths are not used)."""
    bnb = types.ModuleType("bitsandbytes")
    functional = types.ModuleType("bitsandbytes.functional")

    class _Lib:
        def __getattr__(self, name):
            return lambda *a, **k: None

    functional.lib = _Lib()
    functional.QuantState = object
    functional.get_ptr = lambda t: None
    bnb.functional = functional
    sys.modules["bitsandbytes"] = bnb
    sys.modules["bitsandbytes.functional"] = functional
    path = os.path.join(root, "src", "meepsquared", "_vendor", "axolotl", "quantize.py")
    spec = importlib.util.spec_from_file_location("reference_axolotl_quantize", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def bits(t):
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def tile_maps(grouped):
    cases = {}
    cases["kat1"] = ([5, 0, 130, 64], 199, 64)   # tests/test_grouped.py:18-25
    cases["kat2"] = ([0, 0, 7], 7, 64)            # tests/test_grouped.py:28-31
    g = torch.Generator().manual_seed(0)
    for i in range(6):
        experts = int(torch.randint(1, 40, (1,), generator=g))
        counts = torch.randint(0, 300, (experts,), generator=g)
        counts[torch.rand(experts, generator=g) < 0.3] = 0
        cases[f"rand{i}"] = (counts.tolist(), int(counts.sum()), [64, 128][i % 2])
    out = {}
    for name, (counts, rows, block_m) in cases.items():
        offsets = torch.cumsum(torch.tensor(counts, dtype=torch.int32), 0, dtype=torch.int32)
        te, tr, tiles = grouped.tile_map(offsets, rows, block_m)
        out[f"{name}_offsets"] = offsets.numpy()
        out[f"{name}_rows"] = np.array(rows)
        out[f"{name}_block_m"] = np.array(block_m)
        out[f"{name}_tile_expert"] = te.numpy()
        out[f"{name}_tile_row"] = tr.numpy()
        out[f"{name}_tiles"] = np.array(int(tiles))
    return out


def routings():
    """The reference's permutation steps (_moe.py:77-84) on seeded router outputs."""
    out = {}
    for name, (tokens, experts, k, zipf) in {"small": (64, 4, 2, None), "config1": (512, 8, 2, None),
                                             "e128": (2048, 128, 8, None), "zipf": (4096, 128, 8, 1.1)}.items():
        index, _ = layer_inputs.routing(tokens, experts, k, torch.Generator().manual_seed(1), zipf)
        if name == "small":  # two sentinel assignments (ids >= E sort last and are not counted)
            index[3, 1] = experts
            index[40, 0] = experts
        ids = index.reshape(-1)
        ids_g, perm = torch.sort(ids)                       # _moe.py:79, as the reference calls it
        ids_s, perm_s = torch.sort(ids, stable=True)
        hist = torch.histc(ids_g.float(), bins=experts, min=0, max=experts - 1)   # _moe.py:82-83 (CPU branch)
        offsets = torch.cumsum(hist, dim=0, dtype=torch.int32)                     # _moe.py:84
        out[f"{name}_ids"] = ids.numpy()
        out[f"{name}_experts"] = np.array(experts)
        out[f"{name}_perm_reference"] = perm.numpy()
        out[f"{name}_perm_stable"] = perm_s.numpy()
        out[f"{name}_ids_sorted"] = ids_s.numpy()
        out[f"{name}_offsets"] = offsets.numpy()
    return out


def run_layer(moe, cfg, sentinel=False):
    """_moe._routed_forward forward + backward in float32 on a Transformers Qwen3MoeExperts."""
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeExperts

    c = dict(cfg)
    inp = layer_inputs.layer(**c)
    if sentinel:
        inp["top_k_index"][5, 1] = c["experts"]
        inp["top_k_index"][17, 0] = c["experts"]
    conf = Qwen3MoeConfig(hidden_size=c["hidden"], moe_intermediate_size=c["inter"], num_experts=c["experts"],
                          num_experts_per_tok=c["top_k"])
    experts = Qwen3MoeExperts(conf)
    experts.gate_up_proj = torch.nn.Parameter(inp["gate_up"].clone(), requires_grad=False)
    experts.down_proj = torch.nn.Parameter(inp["down"].clone(), requires_grad=False)
    hidden = inp["hidden"].clone().requires_grad_()
    weights = inp["top_k_weights"].clone().requires_grad_()
    leaves = {n: inp[n].clone().requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
               "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}
    os.environ.pop("MEEPSQUARED_GROUPED_KERNEL", None)
    out = moe._routed_forward(experts, hidden, inp["top_k_index"], weights, factors)
    out.backward(inp["grad"])
    res = {"out": out.detach().numpy(), "grad_hidden": hidden.grad.numpy(), "grad_weights": weights.grad.numpy()}
    for n, t in leaves.items():
        res[f"grad_{n}"] = t.grad.numpy()
    return res


def run_layer_bf16(moe, cfg):
    """_moe._routed_forward forward + backward on a bf16 model (a bf16 Qwen3MoeExperts, bf16 hidden states and
    factors, float32 routing weights, bf16 upstream gradient): the reference's bf16 path, every intermediate tensor
    rounded where PyTorch rounds it."""
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeExperts

    c = dict(cfg)
    inp = layer_inputs.layer(**c)
    conf = Qwen3MoeConfig(hidden_size=c["hidden"], moe_intermediate_size=c["inter"], num_experts=c["experts"],
                          num_experts_per_tok=c["top_k"])
    experts = Qwen3MoeExperts(conf).to(torch.bfloat16)
    experts.gate_up_proj = torch.nn.Parameter(inp["gate_up"].to(torch.bfloat16), requires_grad=False)
    experts.down_proj = torch.nn.Parameter(inp["down"].to(torch.bfloat16), requires_grad=False)
    hidden = inp["hidden"].to(torch.bfloat16).requires_grad_()
    weights = inp["top_k_weights"].clone().requires_grad_()
    leaves = {n: inp[n].to(torch.bfloat16).requires_grad_()
              for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
               "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}
    os.environ.pop("MEEPSQUARED_GROUPED_KERNEL", None)
    out = moe._routed_forward(experts, hidden, inp["top_k_index"], weights, factors)
    out.backward(inp["grad"].to(torch.bfloat16))
    res = {"out": bits(out), "grad_hidden": bits(hidden.grad), "grad_weights": weights.grad.numpy()}
    for n, t in leaves.items():  # the adapters' gradients of experts 0, 5, 10 and 15
        res[f"grad_{n}"] = bits(t.grad[::5])
    return res


def fp8_stacks(fp8):
    out = {}
    torch.manual_seed(0)
    stack = torch.randn(4, 6, 8, dtype=torch.bfloat16) * torch.tensor([0.01, 0.1, 1.0, 10.0]).view(4, 1, 1).to(torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    big = (torch.randn(3, 64, 96, generator=g) * 0.05).to(torch.bfloat16)
    big[1, 5, 7] = 3.0  # an outlier sets expert 1's scale
    for name, w in (("test", stack), ("big", big)):
        w8, scale = fp8.quantize_stack(w)
        back = fp8.dequantize_stack(w8, scale, torch.bfloat16)
        out[f"{name}_weight"] = bits(w)
        out[f"{name}_codes"] = w8.view(torch.uint8).numpy()
        out[f"{name}_scale"] = scale.numpy()
        out[f"{name}_dequant"] = bits(back)
    return out


def fp8_blocks(q):
    out = {}
    g = torch.Generator().manual_seed(4)
    for name, (rows, cols) in {"even": (256, 128), "tail": (200, 140)}.items():
        w = layer_inputs.bf16_valued(torch.randn(rows, cols, generator=g) * 0.03)
        w[7, 9] = 1.5
        like = torch.empty(-(-rows // 128), -(-cols // 128), dtype=torch.float32)
        codes, scale_inv = q.quantize_fp8(w, like)
        back = q.dequantize_fp8(codes, scale_inv, torch.bfloat16)
        out[f"{name}_weight"] = bits(w.to(torch.bfloat16))
        out[f"{name}_codes"] = codes.view(torch.uint8).numpy()
        out[f"{name}_scale"] = scale_inv.numpy()
        out[f"{name}_dequant"] = bits(back)
    return out


def grouped_case(grouped):
    """reference_lora forward + backward on the reference tests' ragged case (tests/test_grouped.py:103-143), float32."""
    out = {}
    for is_transposed in (False, True):
        g = torch.Generator().manual_seed(5)
        rows_per_expert = [37, 0, 200, 64, 1]
        K, N, rank = 96, 80, 4
        E = len(rows_per_expert)
        offsets = torch.cumsum(torch.tensor(rows_per_expert, dtype=torch.int32), 0, dtype=torch.int32)
        bv = layer_inputs.bf16_valued
        x = bv(torch.randn(sum(rows_per_expert), K, generator=g)).requires_grad_()
        shape = (E, K, N) if is_transposed else (E, N, K)
        weight = bv(torch.randn(shape, generator=g) * 0.05)
        scale = torch.rand(E, generator=g) + 0.5
        if is_transposed:
            lhs = bv(torch.randn(E, K, rank, generator=g) * 0.1).requires_grad_()
            rhs = bv(torch.randn(E, rank, N, generator=g) * 0.1).requires_grad_()
        else:
            lhs = bv(torch.randn(E, N, rank, generator=g) * 0.1).requires_grad_()
            rhs = bv(torch.randn(E, rank, K, generator=g) * 0.1).requires_grad_()
        bias = bv(torch.randn(E, N, generator=g))
        grad = bv(torch.randn(sum(rows_per_expert), N, generator=g))
        y = grouped.reference_lora(x, weight, scale, offsets, is_transposed, lhs, rhs, 2.0, bias)
        y.backward(grad)
        p = "t_" if is_transposed else "n_"
        for name, t in (("x", x), ("weight", weight), ("lhs", lhs), ("rhs", rhs), ("bias", bias), ("grad", grad)):
            out[p + name] = bits(t.to(torch.bfloat16))  # bf16-valued inputs, stored as bit patterns
        for name, t in (("offsets", offsets), ("scale", scale), ("out", y), ("grad_x", x.grad),
                        ("grad_lhs", lhs.grad), ("grad_rhs", rhs.grad)):
            out[p + name] = t.detach().numpy()
    return out


def merged_stacks(root, fp8):
    """_save._merged_stack (_save.py:79-95) on expert stacks with a PEFT-shaped stand-in for the wrapper (the
    attributes _moe._delta_factors and _save._the_adapter read): bf16 and FP8 stacks, both layouts, bf16 and float32
    outputs."""
    save = importlib.import_module("meepsquared._save")
    out = {}
    g = torch.Generator().manual_seed(6)
    E, rows, cols, rank = 3, 40, 72, 8
    for swapped in (True, False):  # True: the stack is (experts, out, in); False: (experts, in, out)
        p = "n_" if swapped else "t_"
        a = layer_inputs.bf16_valued(torch.randn(E * rank, cols if swapped else rows, generator=g) * 0.2)
        b = layer_inputs.bf16_valued(torch.randn(rows if swapped else cols, rank * E, generator=g) * 0.2)
        wrapper = types.SimpleNamespace(active_adapters=["default"], use_dora={}, num_experts=E,
                                        _did_swap_in_out_features=swapped, scaling={"default": 1.5},
                                        lora_A={"default": types.SimpleNamespace(weight=a)},
                                        lora_B={"default": types.SimpleNamespace(weight=b)})
        stack = layer_inputs.bf16_valued(torch.randn(E, rows, cols, generator=g) * 0.05).to(torch.bfloat16)
        moe = importlib.import_module("meepsquared._moe")
        lhs, rhs, scaling = moe._delta_factors(wrapper, "default", torch.float32)
        out[p + "lhs"], out[p + "rhs"] = lhs.contiguous().numpy(), rhs.contiguous().numpy()
        out[p + "scaling"] = np.array(scaling, dtype=np.float64)
        experts = types.SimpleNamespace(stack=stack)
        out[p + "stack"] = bits(stack)
        out[p + "merged_bf16"] = bits(save._merged_stack(experts, "stack", wrapper, torch.bfloat16))
        out[p + "merged_f32"] = save._merged_stack(experts, "stack", wrapper, torch.float32).numpy()
        w8, scale = fp8.quantize_stack(stack)
        experts8 = types.SimpleNamespace(stack=w8)
        setattr(experts8, "stack" + fp8.STACK_SCALE, scale)
        out[p + "codes"], out[p + "scale"] = w8.view(torch.uint8).numpy(), scale.numpy()
        out[p + "fp8_merged_f32"] = save._merged_stack(experts8, "stack", wrapper, torch.float32).numpy()
        out[p + "fp8_merged_bf16"] = bits(save._merged_stack(experts8, "stack", wrapper, torch.bfloat16))
        out[p + "fp8_alone_f32"] = save._merged_stack(experts8, "stack", None, torch.float32).numpy()
    return out


def main(root):
    moe, grouped, fp8 = import_reference(root)
    q = import_quantize(root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    np.savez_compressed(os.path.join(HERE, "tile_map.npz"), **tile_maps(grouped))
    np.savez_compressed(os.path.join(HERE, "routing.npz"), **routings())
    small = run_layer(moe, layer_inputs.SMALL)
    small.update({f"sentinel_{k}": v for k, v in run_layer(moe, layer_inputs.SMALL, sentinel=True).items()})
    np.savez_compressed(os.path.join(HERE, "layer_small.npz"), **small)
    c1 = run_layer(moe, layer_inputs.CONFIG1)
    keep = {}
    for name, v in c1.items():  # config 1 is large: keep leading slices, a strided sample and the norms
        keep[f"{name}_head"] = v.reshape(-1)[:2048]
        keep[f"{name}_sample"] = v.reshape(-1)[::97]
        keep[f"{name}_norm"] = np.array(np.linalg.norm(v.astype(np.float64)))
    np.savez_compressed(os.path.join(HERE, "layer_config1.npz"), **keep)
    np.savez_compressed(os.path.join(HERE, "layer_bf16.npz"), **run_layer_bf16(moe, LAYER_BF16))
    np.savez_compressed(os.path.join(HERE, "fp8_stack.npz"), **fp8_stacks(fp8))
    np.savez_compressed(os.path.join(HERE, "fp8_block.npz"), **fp8_blocks(q))
    np.savez_compressed(os.path.join(HERE, "grouped.npz"), **grouped_case(grouped))
    np.savez_compressed(os.path.join(HERE, "merged.npz"), **merged_stacks(root, fp8))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <meepsquared checkout>")
    main(sys.argv[1])
