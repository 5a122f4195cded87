"""Minimal stand-ins for bitsandbytes' Linear4bit and peft's LoRA layer, for tests only.

bitsandbytes and peft are not installed in this image. These classes carry exactly the fields the
reference's patches read (solution/nf4.py:114-135, solution/attn.py:276-346): a Linear4bit with a
uint8 packed weight holding a ``quant_state`` and a ``compute_dtype``, and a LoRA layer with
``base_layer``, ``lora_A`` / ``lora_B`` / ``lora_dropout`` ModuleDicts, ``scaling``,
``active_adapters``, ``disable_adapters``, ``merged`` and ``use_dora``. Their unpatched forwards
are the plain math (dequantize with torch ops, linear in the compute dtype; base + B(A(drop(x))) *
scaling), the path the patches replace.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from oracle.nf4 import quantize_nf4


class QuantState:
    def __init__(self, st: dict, device, dtype):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
        self.shape, self.nested, self.blocksize = st["shape"], st["nested"], st["blocksize"]
        self.quant_type, self.dtype = "nf4", dtype
        self.code = t(st["code"])
        self.absmax = t(st["absmax"])
        self.state2 = None
        self.offset = None
        if st["nested"]:
            self.state2 = type("State2", (), {})()
            self.state2.absmax, self.state2.code = t(st["absmax2"]), t(st["code2"])
            self.state2.blocksize = st["blocksize2"]
            self.offset = torch.tensor(float(st["offset"]), device=device)
        self._st = st


class Linear4bit(nn.Module):
    """bitsandbytes.nn.Linear4bit stand-in (nf4, double quant, blocksize 64)."""

    def __init__(self, linear: nn.Linear, compute_dtype, device):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.compute_dtype = compute_dtype
        st = quantize_nf4(linear.weight.detach().float().cpu().numpy())
        w = nn.Parameter(torch.from_numpy(st["packed"]).to(device), requires_grad=False)
        w.quant_state = QuantState(st, device, compute_dtype)
        self.weight = w
        self.bias = (None if linear.bias is None else
                     nn.Parameter(linear.bias.detach().float().to(device), requires_grad=False))

    def dequantized(self):
        from oracle.block import dequant_torch
        return dequant_torch(self.weight.quant_state._st).to(self.weight.device)

    def forward(self, x):
        w = self.dequantized().to(self.compute_dtype)
        b = None if self.bias is None else self.bias.to(self.compute_dtype)
        return F.linear(x.to(self.compute_dtype), w, b).to(x.dtype)


class LoraLayer(nn.Module):
    """peft LoRA Linear stand-in with one adapter named "default"."""

    def __init__(self, base: nn.Module, r: int, alpha: int, dropout: float, device):
        super().__init__()
        self.base_layer = base
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False).to(device)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False).to(device)})
        nn.init.normal_(self.lora_B["default"].weight, std=0.02)
        self.lora_dropout = nn.ModuleDict({"default": nn.Dropout(dropout) if dropout > 0 else nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.active_adapters = ["default"]
        self.disable_adapters = False
        self.merged = False
        self.use_dora = {"default": False}

    def forward(self, x):
        n = "default"
        return self.base_layer(x) + self.lora_B[n](self.lora_A[n](self.lora_dropout[n](x))) * self.scaling[n]
