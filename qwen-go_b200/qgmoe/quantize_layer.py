"""Quantise one raw MoE layer file: the stacked-expert counterpart of qwen-go's
cmd/qwen-quant (which quantises the 2-D linears only, cmd/qwen-quant/
main.go:47-73, 180-213).

    python -m qgmoe.quantize_layer IN OUT --prefix model.layers.3.mlp. --bits 8

reads the raw layer under `prefix` from IN (experts.*.weight stacks in BF16 or
F32, gate.weight, the optional shared expert, as qgmoe_file_layer_desc takes
them), quantises every expert and shared-expert matrix row-wise with the
library's quantizeInt8 / quantizeInt4 on the GPU (bit-exact with the
reference's, model/moe.go:165-217; fp16 scales), and writes the quantised
layer with qgmoe.checkpoint.save_layer (plus quant.json with --quant-json).
"""
from __future__ import annotations

import argparse
import ctypes as C

import numpy as np

from . import DT_BF16, DT_F32, LayerFile
from . import checkpoint as ck


def _array(f: LayerFile, name: str) -> np.ndarray:
    """A tensor of the mapped file as float32 (BF16 widened exactly)."""
    dt, shape, addr, nbytes = f.tensor(name)
    raw = np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(addr)).copy()
    if dt == DT_F32:
        return raw.view(np.float32).reshape(shape)
    if dt == DT_BF16:
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(shape)
    raise ValueError(f"{name}: F32 or BF16 expected")


def quantize_rows_gpu(w: np.ndarray, bits: int, device: int = 0):
    """quantizeInt8 / quantizeInt4 of the rows of w on the GPU: (codes, fp16
    scale bits)."""
    import torch

    from . import quantize_device
    t = torch.from_numpy(np.ascontiguousarray(w, np.float32)).to(f"cuda:{device}")
    q, _, s16 = quantize_device(t, bits)
    return q.cpu().numpy(), s16.cpu().numpy().view(np.uint16)


def quantize_layer(src: str, dst: str, prefix: str, bits: int, quant_json: str | None = None,
                   quantize=None, device: int = 0) -> None:
    quantize = quantize or (lambda w, b: quantize_rows_gpu(w, b, device))
    with LayerFile(src) as f:
        router = _array(f, prefix + "gate.weight")
        E, H = router.shape
        gu = _array(f, prefix + "experts.gate_up_proj.weight")
        dn = _array(f, prefix + "experts.down_proj.weight")
        if gu.ndim != 3 or gu.shape[0] != E or gu.shape[2] != H or dn.shape[:2] != (E, H):
            raise ValueError("expert stacks do not fit the router")
        args = {}
        args["gate_up_q"], args["gate_up_scale"] = quantize(gu.reshape(-1, H), bits)
        args["down_q"], args["down_scale"] = quantize(dn.reshape(E * H, -1), bits)
        try:
            f.tensor(prefix + "shared_expert.gate_proj.weight")
            shared = True
        except Exception:
            shared = False
        if shared:
            for key, base in (("shared_gate", "gate_proj"), ("shared_up", "up_proj"),
                              ("shared_down", "down_proj")):
                w = _array(f, prefix + "shared_expert." + base + ".weight")
                args[key + "_q"], args[key + "_scale"] = quantize(w, bits)
            args["shared_gate"] = _array(f, prefix + "shared_expert_gate.weight").reshape(H)
    ck.save_layer(dst, prefix, router=router, bits=bits, quant_json=quant_json, **args)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("src")
    ap.add_argument("dst")
    ap.add_argument("--prefix", required=True)
    ap.add_argument("--bits", type=int, choices=[8, 4], default=8)
    ap.add_argument("--quant-json")
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args(argv)
    quantize_layer(a.src, a.dst, a.prefix, a.bits, a.quant_json, device=a.device)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
