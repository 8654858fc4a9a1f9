"""GGUF files to device memory, for the MoE path: the reader of the reference's `strata_mlx/gguf.py:63-132`
(header, metadata, tensor directory, aligned data section; split files) and the part of its loader that builds
a MoE layer (`strata_mlx/load.py:259-263, 411-421`), with the bytes going mmap -> pinned host -> HBM unchanged.

Tensors keep the file's bytes: an expert stack `blk.i.ffn_{gate,up,down}_exps.weight` becomes a
`BlockSwitchLinear` over one uint8 device tensor, the shared expert `blk.i.ffn_{gate,up,down}_shexp.weight` a
`BlockMLP` of `BlockLinear`s, the router `blk.i.ffn_gate_inp.weight` and the shared expert's gate
`blk.i.ffn_gate_inp_shexp.weight` float16 matrices. Shapes are in numpy order (the last axis is the one a row
runs along), the reverse of the file's dimension list.
"""

import mmap
import re
import struct
from dataclasses import dataclass

import numpy as np

# GGML type id -> (name, weights per block, bytes per block): the file format's table (the reference's
# strata_mlx/gguf.py:25-33 plus Q2_K, which the B200 path also reads)
TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 30: ("BF16", 1, 2),
    2: ("Q4_0", 32, 18), 6: ("Q5_0", 32, 22), 8: ("Q8_0", 32, 34),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210), 16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98),
    20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110), 22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136),
    29: ("IQ1_M", 256, 56), 42: ("Q2_0", 64, 18),
}
# metadata value type -> struct format (8: string, 9: array are read apart)
_SCALARS = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}


@dataclass
class Tensor:
    name: str
    shape: tuple  # numpy order
    type: str
    data: np.ndarray  # uint8, a view of the file's bytes
    path: str = ""
    offset: int = 0  # where the bytes start in the file

    @property
    def quantized(self) -> bool:
        return self.type not in ("F32", "F16", "BF16")


class _Cursor:
    def __init__(self, buf):
        self.buf, self.at = buf, 0

    def take(self, fmt: str):
        fmt = "<" + fmt
        vals = struct.unpack_from(fmt, self.buf, self.at)
        self.at += struct.calcsize(fmt)
        return vals

    def one(self, fmt: str):
        return self.take(fmt)[0]

    def string(self) -> str:
        n = self.one("Q")
        s = bytes(self.buf[self.at : self.at + n]).decode("utf-8", "replace")
        self.at += n
        return s

    def value(self, vtype: int):
        if vtype == 8:
            return self.string()
        if vtype == 9:
            etype, n = self.take("IQ")
            if etype in _SCALARS:  # one unpack for the whole array
                vals = self.take(f"{n}{_SCALARS[etype]}")
                return list(vals)
            return [self.value(etype) for _ in range(n)]
        if vtype not in _SCALARS:
            raise ValueError(f"GGUF metadata value type {vtype} is not known")
        return self.one(_SCALARS[vtype])


class GGUF:
    """One GGUF file, memory-mapped: `meta` (key -> value) and `tensors` (name -> Tensor over the map)."""

    def __init__(self, path: str):
        self.path = path
        self._file = open(path, "rb")
        self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        c = _Cursor(self._map)
        if bytes(self._map[:4]) != b"GGUF":
            raise ValueError(f"{path} is not a GGUF file")
        c.at = 4
        self.version, n_tensors, n_kv = c.take("IQQ")
        if self.version < 2:
            raise ValueError(f"{path}: GGUF version {self.version} is not supported")
        self.meta = {}
        for _ in range(n_kv):
            key = c.string()
            self.meta[key] = c.value(c.one("I"))
        directory = []
        for _ in range(n_tensors):
            name = c.string()
            dims = c.take(f"{c.one('I')}Q")
            type_id, offset = c.take("IQ")
            directory.append((name, tuple(int(d) for d in reversed(dims)), type_id, offset))
        align = int(self.meta.get("general.alignment", 32))
        base = (c.at + align - 1) // align * align
        raw = np.frombuffer(self._map, dtype=np.uint8)
        self.tensors = {}
        for name, shape, type_id, offset in directory:
            if type_id not in TYPES:
                raise ValueError(f"{name}: GGUF tensor type {type_id} is not supported")
            kind, per, nbytes = TYPES[type_id]
            count = int(np.prod(shape, dtype=np.int64))
            if count % per:
                raise ValueError(f"{name}: {count} weights do not fill {kind} blocks of {per}")
            n = count // per * nbytes
            at = base + offset
            if at + n > raw.size:
                raise ValueError(f"{name}: its bytes run past the end of {path}")
            self.tensors[name] = Tensor(name, shape, kind, raw[at : at + n], path, at)

    def __getitem__(self, name: str) -> Tensor:
        return self.tensors[name]

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def close(self) -> None:
        self.tensors = {}
        try:
            self._map.close()
        except BufferError:
            pass  # views of its bytes are still held elsewhere: the map goes with the last of them
        self._file.close()


_SPLIT = re.compile(r"-(\d{5})-of-(\d{5})\.gguf$")


def shards(path: str) -> list:
    """A model's files: the one named and, where its name says it is one of several (`-00001-of-00003.gguf`),
    the others beside it (strata_mlx/gguf.py:135-140)."""
    m = _SPLIT.search(path)
    count = int(m.group(2)) if m else 1
    return [GGUF(path)] + [GGUF(_SPLIT.sub(f"-{i:05d}-of-{m.group(2)}.gguf", path)) for i in range(2, count + 1)]


def find(files: list, name: str) -> Tensor:
    for f in files:
        if name in f:
            return f[name]
    raise KeyError(f"{name} is in none of the model's files")


# ---------------------------------------------------------------- to the device

UPLOAD_CHUNK = 64 << 20  # bytes a pinned staging buffer holds


def to_device(data: np.ndarray, device) -> "torch.Tensor":
    """A uint8 copy of `data` (a view of a mapped file) on `device`. To a GPU the bytes go through two pinned
    staging buffers of UPLOAD_CHUNK bytes in turn: the host copies chunk i + 1 from the map while chunk i
    travels on a side stream; on the CPU a plain copy."""
    import torch

    flat = np.ascontiguousarray(data).reshape(-1)
    device = torch.device(device)
    if device.type != "cuda":
        return torch.from_numpy(flat.copy())
    out = torch.empty(flat.size, dtype=torch.uint8, device=device)
    if flat.size == 0:
        return out
    n = min(UPLOAD_CHUNK, flat.size)
    staging = [torch.empty(n, dtype=torch.uint8).pin_memory() for _ in range(2)]
    done = [None, None]
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))  # (out's memory may have been in use on that stream)
    for i, at in enumerate(range(0, flat.size, n)):
        b = i & 1
        if done[b] is not None:
            done[b].synchronize()  # the copy that last used this buffer has left it
        m = min(n, flat.size - at)
        staging[b][:m].numpy()[:] = flat[at : at + m]
        with torch.cuda.stream(side):
            out[at : at + m].copy_(staging[b][:m], non_blocking=True)
            done[b] = torch.cuda.Event()
            done[b].record(side)
    side.synchronize()
    return out


def float_matrix(t: Tensor, device, dtype=None) -> "torch.Tensor":
    """A float tensor (F32, F16, BF16) of the file as a device matrix in `dtype` (float16 by default)."""
    import torch

    if t.type == "F32":
        w = torch.from_numpy(t.data.view(np.float32).reshape(t.shape).copy())
    elif t.type == "F16":
        w = torch.from_numpy(t.data.view(np.float16).reshape(t.shape).copy())
    elif t.type == "BF16":
        w = torch.from_numpy(t.data.view(np.int16).reshape(t.shape).copy()).view(torch.bfloat16)
    else:
        raise ValueError(f"{t.name}: {t.type} is not a float type")
    return w.to(device=device, dtype=dtype or torch.float16)


def experts(t: Tensor, device):
    """A stack of experts (E, rows, cols), kept as the file's blocks (strata_mlx/load.py:259-263)."""
    from .blocks import BLOCK, BlockSwitchLinear

    if t.type not in BLOCK:
        raise ValueError(f"{t.name}: {t.type} experts are not supported")
    if len(t.shape) != 3:
        raise ValueError(f"{t.name}: an expert stack has three axes, not {len(t.shape)}")
    return BlockSwitchLinear(to_device(t.data, device), t.type, t.shape)


def linear(t: Tensor, device):
    """One matrix (rows, cols) kept as the file's blocks."""
    from .blocks import BLOCK, BlockLinear

    if t.type not in BLOCK:
        raise ValueError(f"{t.name}: {t.type} matrices are not read as blocks here")
    if len(t.shape) != 2:
        raise ValueError(f"{t.name}: a matrix has two axes, not {len(t.shape)}")
    return BlockLinear(to_device(t.data, device), t.type, t.shape)


def moe_layer(files: list, layer: int, top_k: int | None = None, device="cuda"):
    """Layer `layer`'s MoE block from the model's files (strata_mlx/load.py:411-421): the router, the routed
    experts' three stacks, the shared expert and its gate. `top_k` defaults to the file's
    `<arch>.expert_used_count`."""
    from .blocks import BlockMLP, BlockSwitchGLU
    from .fused import SparseMoeBlock

    b = f"blk.{layer}."
    if top_k is None:
        arch = files[0].meta.get("general.architecture", "")
        top_k = files[0].meta.get(f"{arch}.expert_used_count")
        if top_k is None:
            raise ValueError("top_k is not given and the file does not name the experts used per token")
    router = float_matrix(find(files, b + "ffn_gate_inp.weight"), device)
    sgate = float_matrix(find(files, b + "ffn_gate_inp_shexp.weight"), device).reshape(1, -1)
    switch = BlockSwitchGLU(*(experts(find(files, b + f"ffn_{p}_exps.weight"), device) for p in ("gate", "up", "down")))
    shared = BlockMLP(*(linear(find(files, b + f"ffn_{p}_shexp.weight"), device) for p in ("gate", "up", "down")))
    return SparseMoeBlock(router, switch, shared, sgate, int(top_k))


_EXPERT_LAYER = re.compile(r"^blk\.(\d+)\.ffn_gate_exps\.weight$")


def moe_layers(files: list, top_k: int | None = None, device="cuda") -> dict:
    """Every MoE layer of the model's files: layer index -> SparseMoeBlock (the layers whose routed experts'
    gate stack is in the files), uploaded one layer at a time."""
    found = sorted({int(m.group(1)) for f in files for name in f.tensors if (m := _EXPERT_LAYER.match(name))})
    return {i: moe_layer(files, i, top_k, device) for i in found}


__all__ = ["GGUF", "TYPES", "Tensor", "experts", "find", "float_matrix", "linear", "moe_layer", "moe_layers",
           "shards", "to_device"]
