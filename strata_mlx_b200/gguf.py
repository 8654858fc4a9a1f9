"""GGUF files to device memory, for the MoE path: a reader of the container (header, metadata, tensor
directory, aligned data section; split files) that serves what the reference's `strata_mlx/gguf.py:63-132`
serves, and the part of its loader that builds a MoE layer (`strata_mlx/load.py:259-263, 411-421`), with the
bytes going mmap -> pinned host -> HBM unchanged.

Tensors keep the file's bytes: an expert stack `blk.i.ffn_{gate,up,down}_exps.weight` becomes a
`BlockSwitchLinear` over one uint8 device tensor, the shared expert `blk.i.ffn_{gate,up,down}_shexp.weight` a
`BlockMLP` of `BlockLinear`s, the router `blk.i.ffn_gate_inp.weight` and the shared expert's gate
`blk.i.ffn_gate_inp_shexp.weight` float16 matrices. Shapes are given in numpy order, slowest axis first: the
file lists them fastest first, so they are reversed on reading.
"""

import mmap
import os
import re
from dataclasses import dataclass

import numpy as np

# GGML type id -> (name, weights per block, bytes per block): the file format's table of tensor types (the
# reference's strata_mlx/gguf.py:25-33 plus Q2_K, which the B200 path also reads)
TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 30: ("BF16", 1, 2),
    2: ("Q4_0", 32, 18), 6: ("Q5_0", 32, 22), 8: ("Q8_0", 32, 34),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210), 16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98),
    20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110), 22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136),
    29: ("IQ1_M", 256, 56), 42: ("Q2_0", 64, 18),
}

MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32  # the data section's alignment when the file does not name one (`general.alignment`)
# metadata value types of the format: the fixed-size ones as numpy dtypes; 8 is a string, 9 an array
VALUE_DTYPES = {0: np.dtype("<u1"), 1: np.dtype("<i1"), 2: np.dtype("<u2"), 3: np.dtype("<i2"), 4: np.dtype("<u4"),
                5: np.dtype("<i4"), 6: np.dtype("<f4"), 7: np.dtype("?"), 10: np.dtype("<u8"), 11: np.dtype("<i8"),
                12: np.dtype("<f8")}
STRING, ARRAY = 8, 9


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


class _Fields:
    """Little-endian fields read off a byte buffer one after the other (numpy views, no copies of arrays)."""

    __slots__ = ("buf", "pos", "path")

    def __init__(self, buf, pos: int, path: str):
        self.buf, self.pos, self.path = buf, pos, path

    def numbers(self, dtype: np.dtype, count: int) -> np.ndarray:
        end = self.pos + dtype.itemsize * count
        if end > len(self.buf):
            raise ValueError(f"{self.path}: the header runs past the end of the file")
        out = np.frombuffer(self.buf, dtype=dtype, count=count, offset=self.pos)
        self.pos = end
        return out

    def number(self, dtype: np.dtype):
        return self.numbers(dtype, 1)[0].item()

    def text(self) -> str:
        n = self.number(VALUE_DTYPES[10])
        raw = self.numbers(np.dtype("u1"), n)
        return raw.tobytes().decode("utf-8", errors="replace")

    def value(self, vtype: int):
        if vtype in VALUE_DTYPES:
            return self.number(VALUE_DTYPES[vtype])
        if vtype == STRING:
            return self.text()
        if vtype == ARRAY:
            etype = self.number(VALUE_DTYPES[4])
            count = self.number(VALUE_DTYPES[10])
            if etype in VALUE_DTYPES:
                return self.numbers(VALUE_DTYPES[etype], count).tolist()
            return [self.value(etype) for _ in range(count)]
        raise ValueError(f"{self.path}: metadata value of unknown type {vtype}")


def read_header(buf, path: str = ""):
    """(version, metadata dict, [(name, numpy-order shape, type id, offset in the data section)], where the data
    section starts) of a GGUF file's bytes. The header is: magic, version u32, tensor count u64, metadata count
    u64; the metadata (string key, u32 value type, value); per tensor its string name, u32 axis count, u64 axes
    (fastest first), u32 type, u64 offset; then the data section, aligned."""
    if len(buf) < 24 or bytes(buf[:4]) != MAGIC:
        raise ValueError(f"{path}: no GGUF magic at the start; not a GGUF file")
    f = _Fields(buf, 4, path)
    version = f.number(VALUE_DTYPES[4])
    if version < 2:
        raise ValueError(f"{path}: GGUF version {version} predates the 64-bit header this reader takes")
    n_tensors, n_meta = (int(v) for v in f.numbers(VALUE_DTYPES[10], 2))
    meta = {}
    for _ in range(n_meta):
        key = f.text()
        meta[key] = f.value(f.number(VALUE_DTYPES[4]))
    entries = []
    for _ in range(n_tensors):
        name = f.text()
        axes = f.numbers(VALUE_DTYPES[10], f.number(VALUE_DTYPES[4]))
        type_id = f.number(VALUE_DTYPES[4])
        offset = f.number(VALUE_DTYPES[10])
        entries.append((name, tuple(int(a) for a in axes[::-1]), type_id, offset))
    align = int(meta.get("general.alignment", DEFAULT_ALIGNMENT))
    start = -(-f.pos // align) * align
    return version, meta, entries, start


class GGUF:
    """One GGUF file, memory-mapped: `meta` (key -> value) and `tensors` (name -> Tensor over the map)."""

    def __init__(self, path: str):
        self.path = path
        self._file = open(path, "rb")
        self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            self.version, self.meta, entries, start = read_header(self._map, path)
            raw = np.frombuffer(self._map, dtype=np.uint8)
            self.tensors = {}
            for name, shape, type_id, offset in entries:
                self.tensors[name] = _tensor(raw, path, name, shape, type_id, start + offset)
        except Exception:
            self.close()
            raise

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


def _tensor(raw: np.ndarray, path: str, name: str, shape: tuple, type_id: int, at: int) -> Tensor:
    if type_id not in TYPES:
        raise ValueError(f"{path}: tensor {name} has GGML type {type_id}, which this reader does not know")
    kind, per, nbytes = TYPES[type_id]
    weights = int(np.prod(shape, dtype=np.int64))
    blocks, rest = divmod(weights, per)
    if rest:
        raise ValueError(f"{path}: tensor {name} of {weights} weights is not whole {kind} blocks of {per}")
    end = at + blocks * nbytes
    if end > raw.size:
        raise ValueError(f"{path}: tensor {name} ends {end - raw.size} bytes past the end of the file")
    return Tensor(name, shape, kind, raw[at:end], path, at)


def _numbered(path: str):
    """(prefix, number, count) of a file named `<prefix>-<number>-of-<count>.gguf` (five digits each), else None."""
    stem = os.path.basename(path)
    if not stem.endswith(".gguf"):
        return None
    parts = stem[: -len(".gguf")].rsplit("-", 3)
    if len(parts) != 4 or parts[2] != "of" or not (len(parts[1]) == len(parts[3]) == 5):
        return None
    if not (parts[1].isdigit() and parts[3].isdigit()):
        return None
    return os.path.join(os.path.dirname(path), parts[0]), int(parts[1]), int(parts[3])


def shards(path: str) -> list:
    """Open every file of a model given its first file's path, in split order. The split is the file's
    `split.count` (with `split.no` its own place, from 0) where it has them, else what its name says
    (`<prefix>-00001-of-00003.gguf`); the other files are the same prefix with their numbers."""
    first = GGUF(path)
    count = first.meta.get("split.count")
    named = _numbered(path)
    if count is None:
        count = named[2] if named else 1
    count = int(count)
    if count <= 1:
        return [first]
    if named is None:
        first.close()
        raise ValueError(f"{path}: a split of {count} files, but the name does not number it")
    prefix, _, _ = named
    files = [first]
    for i in range(2, count + 1):
        f = GGUF(f"{prefix}-{i:05d}-of-{count:05d}.gguf")
        no = f.meta.get("split.no")
        if no is not None and int(no) != i - 1:
            raise ValueError(f"{f.path}: split.no is {no}, not {i - 1}")
        files.append(f)
    return files


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
        raise ValueError(f"{t.name}: no block kernel reads {t.type} expert stacks")
    if len(t.shape) != 3:
        raise ValueError(f"{t.name}: an expert stack has three axes, not {len(t.shape)}")
    return BlockSwitchLinear(to_device(t.data, device), t.type, t.shape)


def linear(t: Tensor, device):
    """One matrix (rows, cols) kept as the file's blocks."""
    from .blocks import BLOCK, BlockLinear

    if t.type not in BLOCK:
        raise ValueError(f"{t.name}: no block kernel reads {t.type} matrices")
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
