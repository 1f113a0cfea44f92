"""FerrisRes checkpoint ingestion for the ternary MoE layers.

A FerrisRes checkpoint is a safetensors file plus a JSON config
(src/model/checkpoint.rs:1-29).  The MoE tensors of layer i are
``layers.{i}.moe.router`` [num_experts, hidden] and
``layers.{i}.moe.expert.{e}.{gate,up,down}`` ([inter, hidden] /
[hidden, inter]), stored as BF16 or F32; the reference loads them as fp32
(get_tensor_f32, src/model/safetensors.rs:88-129) and re-quantizes every
expert matrix with TernaryExpert::from_fp32 (src/model/checkpoint.rs:387-400).
Here the file is memory-mapped, each matrix is widened to fp32 exactly as the
reference does (BF16: the upper half of an fp32), and quantized on the device
by ``ft_moe_create_f32`` straight into the resident layout.

The safetensors reader follows the published format: an 8-byte little-endian
header length, a JSON header of {name: {dtype, shape, data_offsets}}, then
the raw little-endian tensor bytes.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

from ._lib import ShapeError, UnsupportedError

_NP = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I8": np.int8, "U8": np.uint8,
       "I16": np.int16, "I32": np.int32, "I64": np.int64}


class SafeTensors:
    """A memory-mapped safetensors file."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        self.meta = header.pop("__metadata__", {})
        self.header = header
        self._data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)

    def names(self):
        return list(self.header)

    def info(self, name: str):
        if name not in self.header:
            raise ShapeError(f"tensor '{name}' not found in {self.path}")
        h = self.header[name]
        return h["dtype"], tuple(h["shape"])

    def raw(self, name: str) -> np.ndarray:
        dtype, shape = self.info(name)
        if dtype not in _NP:
            raise UnsupportedError(f"unsupported safetensors dtype {dtype}")
        b, e = self.header[name]["data_offsets"]
        a = self._data[b:e].view(np.dtype(_NP[dtype]).newbyteorder("<"))
        if a.size != int(np.prod(shape)):
            raise ShapeError(f"tensor '{name}': {a.size} elements for shape {shape}")
        return a.reshape(shape)

    def get_f32(self, name: str) -> np.ndarray:
        """The tensor widened to fp32 (src/model/safetensors.rs:88-129: BF16 is
        the upper 16 bits of an fp32, F16 the IEEE half)."""
        dtype, _ = self.info(name)
        a = self.raw(name)
        if dtype == "F32":
            return np.ascontiguousarray(a, np.float32)
        if dtype == "BF16":
            return (a.astype(np.uint32) << 16).view(np.float32)
        if dtype == "F16":
            return a.astype(np.float32)
        raise UnsupportedError(f"cannot widen dtype {dtype} to f32")


def f32_to_bf16_bits(a) -> np.ndarray:
    """The reference writer's BF16 (src/model/safetensors.rs:616-620): the upper
    16 bits of the fp32 pattern (truncation)."""
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def write_safetensors(path: str, tensors) -> None:
    """Writes {name: (array, dtype)} (dtype "F32" or "BF16") in the layout of the
    reference writer (src/model/safetensors.rs:628-680): tensors in the given
    order, header {dtype, shape, data_offsets}."""
    header, blobs, off = {}, [], 0
    for name, (arr, dtype) in tensors.items():
        a = np.asarray(arr, np.float32)
        data = (f32_to_bf16_bits(a) if dtype == "BF16" else a).astype(
            np.uint16 if dtype == "BF16" else np.float32).tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def load_config(path: str) -> dict:
    """The model JSON (BlockMoeResConfig, src/model/checkpoint.rs:37-70)."""
    with open(path) as f:
        return json.load(f)


def load_moe_layer(st, layer: int, top_k: int = 2, use_gelu: bool = False, device=None,
                   rank: int = 0, world: int = 1):
    """The MoE layer ``layer`` of an open SafeTensors file as a resident
    TernaryMoELayer.  With world > 1 only experts [rank*E/world, (rank+1)*E/world)
    are read and uploaded (expert parallelism; the router is always complete)."""
    from .moe import TernaryMoELayer
    pfx = f"layers.{layer}.moe"
    router = st.get_f32(f"{pfx}.router")
    if router.ndim != 2:
        raise ShapeError(f"{pfx}.router must be [num_experts, hidden]")
    E, H = router.shape
    _, gshape = st.info(f"{pfx}.expert.0.gate")
    F = gshape[0]
    if E % world:
        raise ShapeError(f"{E} experts do not split over {world} ranks")
    per = E // world
    mine = range(rank * per, (rank + 1) * per)
    gate, up, down = [], [], []
    for e in range(E):
        if e not in mine:
            gate.append(None), up.append(None), down.append(None)
            continue
        for lst, nm, shape in ((gate, "gate", (F, H)), (up, "up", (F, H)), (down, "down", (H, F))):
            a = st.get_f32(f"{pfx}.expert.{e}.{nm}")
            if a.shape != shape:
                raise ShapeError(f"{pfx}.expert.{e}.{nm} has shape {a.shape}, expected {shape}")
            lst.append(a)
    return TernaryMoELayer.from_fp32(router.ravel(), gate, up, down, H, F, top_k, use_gelu, device)


def load_moe_layers(path: str, device=None, rank: int = 0, world: int = 1):
    """Every MoE layer of the checkpoint ``{path}.safetensors`` + ``{path}.json``
    (load_model's MoE branch, src/model/checkpoint.rs:388-417), as
    {layer index: TernaryMoELayer}."""
    cfg = load_config(f"{path}.json")
    st = SafeTensors(f"{path}.safetensors")
    layers = {}
    for i, lc in enumerate(cfg.get("layer_configs", [])):
        if not lc.get("has_moe"):
            continue
        layers[i] = load_moe_layer(st, i, int(lc.get("top_k", 2)), bool(lc.get("use_gelu", False)),
                                   device, rank, world)
        if layers[i].n_experts != int(lc.get("num_experts", layers[i].n_experts)) or \
                layers[i].intermediate_dim != int(lc.get("inter_dim", layers[i].intermediate_dim)):
            raise ShapeError(f"layer {i}: tensors disagree with the config")
    return layers
