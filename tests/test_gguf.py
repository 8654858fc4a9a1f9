"""The GGUF reader and the MoE layer loader on the host (no GPU): files written by gguf-py 0.19.0's own writer
(the version the reference pins) read back, metadata, shapes in numpy order, types and the bytes of every
tensor; split files; the layer's structure built on the CPU (strata_mlx/gguf.py:63-140,
strata_mlx/load.py:411-421)."""

import numpy as np
import pytest

gguf_py = pytest.importorskip("gguf")
torch = pytest.importorskip("torch")

from oracle import quants as Q  # noqa: E402
from strata_mlx_b200 import gguf as G  # noqa: E402

H, F_, E, FS, K = 512, 256, 8, 512, 2


def write(path, tensors, meta=None, arch="test"):
    """tensors: name -> (array, ggml type name or None for float arrays); block types given as uint8 bytes
    (experts, rows, bytes a row), the logical shape worked out by the writer."""
    w = gguf_py.GGUFWriter(str(path), arch)
    w.add_uint32(f"{arch}.expert_used_count", K)
    for key, value in (meta or {}).items():
        if isinstance(value, str):
            w.add_string(key, value)
        elif isinstance(value, float):
            w.add_float32(key, value)
        elif isinstance(value, list) and value and isinstance(value[0], str):
            w.add_array(key, value)
        elif isinstance(value, list):
            w.add_array(key, value)
        else:
            w.add_uint64(key, value)
    for name, (arr, kind) in tensors.items():
        if kind is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf_py.GGMLQuantizationType[kind])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def stack_bytes(kind, experts, rows, cols, rng):
    per, nbytes = Q.TYPES[kind][1], Q.TYPES[kind][2]
    b = Q.random_blocks(kind, experts * rows * cols // per, rng, normal=0.001)
    return b.reshape(experts, rows, cols // per * nbytes) if experts > 1 else b.reshape(rows, cols // per * nbytes)


def layer_tensors(rng, layer=0, kinds=("IQ3_S", "IQ3_S", "Q2_K"), shared="Q8_0"):
    b = f"blk.{layer}."
    return {
        b + "ffn_gate_inp.weight": ((0.02 * rng.standard_normal((E, H))).astype(np.float32), None),
        b + "ffn_gate_inp_shexp.weight": ((0.02 * rng.standard_normal(H)).astype(np.float32), None),
        b + "ffn_gate_exps.weight": (stack_bytes(kinds[0], E, F_, H, rng), kinds[0]),
        b + "ffn_up_exps.weight": (stack_bytes(kinds[1], E, F_, H, rng), kinds[1]),
        b + "ffn_down_exps.weight": (stack_bytes(kinds[2], E, H, F_, rng), kinds[2]),
        b + "ffn_gate_shexp.weight": (stack_bytes(shared, 1, FS, H, rng), shared),
        b + "ffn_up_shexp.weight": (stack_bytes(shared, 1, FS, H, rng), shared),
        b + "ffn_down_shexp.weight": (stack_bytes(shared, 1, H, FS, rng), shared),
    }


def test_a_file_reads_back_what_was_written(tmp_path):
    rng = np.random.default_rng(0)
    tensors = layer_tensors(rng)
    tensors["token_embd.weight"] = (rng.standard_normal((16, H)).astype(np.float16), None)
    meta = {"general.name": "tiny", "test.rope.freq_base": 0.5, "test.ids": [3, 1, 4, 1, 5],
            "tokenizer.ggml.tokens": ["a", "bb", "ccc"], "test.context_length": 4096}
    path = tmp_path / "tiny.gguf"
    write(path, tensors, meta)
    f = G.GGUF(str(path))
    assert f.meta["general.name"] == "tiny" and f.meta["general.architecture"] == "test"
    assert f.meta["test.expert_used_count"] == K and f.meta["test.context_length"] == 4096
    assert f.meta["test.rope.freq_base"] == pytest.approx(0.5)
    assert f.meta["test.ids"] == [3, 1, 4, 1, 5] and f.meta["tokenizer.ggml.tokens"] == ["a", "bb", "ccc"]
    want_shapes = {"blk.0.ffn_gate_exps.weight": (E, F_, H), "blk.0.ffn_down_exps.weight": (E, H, F_),
                   "blk.0.ffn_gate_shexp.weight": (FS, H), "blk.0.ffn_gate_inp.weight": (E, H),
                   "blk.0.ffn_gate_inp_shexp.weight": (H,), "token_embd.weight": (16, H)}
    for name, shape in want_shapes.items():
        assert f[name].shape == shape, name
    for name, (arr, kind) in tensors.items():
        t = f[name]
        assert t.type == (kind or {np.float32: "F32", np.float16: "F16"}[arr.dtype.type])
        np.testing.assert_array_equal(t.data, arr.reshape(-1).view(np.uint8))
        assert t.quantized == (kind is not None)
    f.close()


def test_split_files_are_found_beside_the_first(tmp_path):
    rng = np.random.default_rng(1)
    tensors = layer_tensors(rng, 0)
    tensors.update(layer_tensors(rng, 1))
    names = sorted(tensors)
    write(tmp_path / "m-00001-of-00002.gguf", {n: tensors[n] for n in names[: len(names) // 2]})
    write(tmp_path / "m-00002-of-00002.gguf", {n: tensors[n] for n in names[len(names) // 2 :]})
    files = G.shards(str(tmp_path / "m-00001-of-00002.gguf"))
    assert len(files) == 2
    for n in names:
        np.testing.assert_array_equal(G.find(files, n).data, tensors[n][0].reshape(-1).view(np.uint8))
    with pytest.raises(KeyError):
        G.find(files, "blk.9.ffn_up_exps.weight")


def test_a_split_is_read_from_its_metadata(tmp_path):
    """split.count / split.no (as llama.cpp's gguf-split writes them) say how many files there are; a file whose
    split.no is not its place in the numbering is refused."""
    rng = np.random.default_rng(4)
    tensors = layer_tensors(rng, 0)
    names = sorted(tensors)
    thirds = [names[:3], names[3:6], names[6:]]
    for i, part in enumerate(thirds):
        write(tmp_path / f"q-{i + 1:05d}-of-00003.gguf", {n: tensors[n] for n in part},
              {"split.no": i, "split.count": 3})
    files = G.shards(str(tmp_path / "q-00001-of-00003.gguf"))
    assert [f.meta["split.no"] for f in files] == [0, 1, 2]
    for n in names:
        np.testing.assert_array_equal(G.find(files, n).data, tensors[n][0].reshape(-1).view(np.uint8))
    write(tmp_path / "r-00001-of-00002.gguf", {names[0]: tensors[names[0]]}, {"split.no": 0, "split.count": 2})
    write(tmp_path / "r-00002-of-00002.gguf", {names[1]: tensors[names[1]]}, {"split.no": 0, "split.count": 2})
    with pytest.raises(ValueError, match="split.no"):
        G.shards(str(tmp_path / "r-00001-of-00002.gguf"))
    # a lone file is its own split
    write(tmp_path / "lone.gguf", {names[0]: tensors[names[0]]})
    assert len(G.shards(str(tmp_path / "lone.gguf"))) == 1


def test_a_truncated_header_is_refused(tmp_path):
    rng = np.random.default_rng(8)
    write(tmp_path / "t.gguf", layer_tensors(rng, 0))
    data = (tmp_path / "t.gguf").read_bytes()
    (tmp_path / "cut.gguf").write_bytes(data[:200])
    with pytest.raises(ValueError):
        G.GGUF(str(tmp_path / "cut.gguf"))


def test_a_moe_layer_is_built_from_the_files_bytes(tmp_path):
    rng = np.random.default_rng(2)
    tensors = layer_tensors(rng, 3, kinds=("Q4_K", "IQ4_XS", "Q6_K"))
    write(tmp_path / "l.gguf", tensors)
    block = G.moe_layer([G.GGUF(str(tmp_path / "l.gguf"))], 3, device="cpu")
    assert block.top_k == K
    sw, sh = block.switch_mlp, block.shared_expert
    for lin, part, kind, shape in ((sw.gate_proj, "gate", "Q4_K", (E, F_, H)), (sw.up_proj, "up", "IQ4_XS", (E, F_, H)),
                                   (sw.down_proj, "down", "Q6_K", (E, H, F_))):
        assert lin.kind == kind and lin.shape == shape
        np.testing.assert_array_equal(lin.blocks.numpy(), tensors[f"blk.3.ffn_{part}_exps.weight"][0].reshape(-1))
    assert (sh.gate_proj.kind, sh.gate_proj.output_dims, sh.gate_proj.input_dims) == ("Q8_0", FS, H)
    assert (sh.down_proj.output_dims, sh.down_proj.input_dims) == (H, FS)
    router = tensors["blk.3.ffn_gate_inp.weight"][0]
    np.testing.assert_array_equal(block.gate.weight.numpy(), router.astype(np.float16))
    assert block.shared_expert_gate.weight.shape == (1, H)


def test_every_moe_layer_of_split_files_is_found(tmp_path):
    rng = np.random.default_rng(5)
    tensors = layer_tensors(rng, 0)
    tensors.update(layer_tensors(rng, 2, kinds=("Q2_K", "Q3_K", "IQ3_XXS")))
    tensors["token_embd.weight"] = (rng.standard_normal((16, H)).astype(np.float16), None)
    names = sorted(tensors)
    write(tmp_path / "s-00001-of-00002.gguf", {n: tensors[n] for n in names[:5]})
    write(tmp_path / "s-00002-of-00002.gguf", {n: tensors[n] for n in names[5:]})
    layers = G.moe_layers(G.shards(str(tmp_path / "s-00001-of-00002.gguf")), device="cpu")
    assert sorted(layers) == [0, 2]
    assert layers[2].switch_mlp.up_proj.kind == "Q3_K" and layers[0].switch_mlp.down_proj.kind == "Q2_K"
    np.testing.assert_array_equal(layers[2].switch_mlp.down_proj.blocks.numpy(),
                                  tensors["blk.2.ffn_down_exps.weight"][0].reshape(-1))


def test_what_is_not_a_gguf_file_or_not_a_block_type_is_refused(tmp_path):
    p = tmp_path / "no.gguf"
    p.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(ValueError):
        G.GGUF(str(p))
    rng = np.random.default_rng(3)
    write(tmp_path / "f.gguf", {"blk.0.ffn_up_exps.weight": (rng.standard_normal((E, F_, H)).astype(np.float16), None)})
    with pytest.raises(ValueError):
        G.experts(G.GGUF(str(tmp_path / "f.gguf"))["blk.0.ffn_up_exps.weight"], "cpu")


@pytest.mark.gpu
def test_a_layer_loaded_to_the_gpu_is_the_layer_built_from_the_same_bytes(cuda, tmp_path, monkeypatch):
    """Through pinned staging buffers (a small chunk, so every tensor takes several and an odd last one) the
    device holds the file's bytes, and the loaded block's output is the directly built block's, bit for bit."""
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as F

    monkeypatch.setattr(G, "UPLOAD_CHUNK", 4096 + 16)
    rng = np.random.default_rng(4)
    tensors = layer_tensors(rng, 0, kinds=("IQ3_S", "IQ3_S", "IQ3_S"))
    write(tmp_path / "g.gguf", tensors)
    files = [G.GGUF(str(tmp_path / "g.gguf"))]
    loaded = G.moe_layer(files, 0, device=cuda)
    for part in ("gate", "up", "down"):
        got = getattr(loaded.switch_mlp, f"{part}_proj").blocks.cpu().numpy()
        np.testing.assert_array_equal(got, tensors[f"blk.0.ffn_{part}_exps.weight"][0].reshape(-1))

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)

    t = {n: a for n, (a, _) in tensors.items()}
    sw = B.BlockSwitchGLU(*(B.BlockSwitchLinear(dev(t[f"blk.0.ffn_{p}_exps.weight"]).reshape(-1), "IQ3_S", s)
                            for p, s in (("gate", (E, F_, H)), ("up", (E, F_, H)), ("down", (E, H, F_)))))
    sh = B.BlockMLP(*(B.BlockLinear(dev(t[f"blk.0.ffn_{p}_shexp.weight"]).reshape(-1), "Q8_0", s)
                      for p, s in (("gate", (FS, H)), ("up", (FS, H)), ("down", (H, FS)))))
    direct = F.SparseMoeBlock(dev(t["blk.0.ffn_gate_inp.weight"].astype(np.float16)), sw, sh,
                              dev(t["blk.0.ffn_gate_inp_shexp.weight"].astype(np.float16).reshape(1, H)), K)
    x = dev(rng.standard_normal((3, H)).astype(np.float16))
    assert torch.equal(loaded(x), direct(x))
