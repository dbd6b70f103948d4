"""CPU: the library's safetensors reader (csrc/st_loader.cu) on checkpoints written in the MLX layout the
reference loads (engine/src/model.c:52-70, engine/src/io/k3_st.c): one or several shards, header checks,
and the no-GPU refusal of qe_moe_open_safetensors."""
import numpy as np
import pytest
import torch

import oracle as O
import qmoe
from golden_io import checkpoint_tensors, write_safetensors

CFG = dict(hidden=256, E=16, top_k=4, inter=64, sh_inter=128, bits=4)
PREFIX = "language_model.model.layers.3.mlp"


def _arrays():
    blk = O.SynthBlock(O.BlockCfg(**CFG, quant_router=True), 21)
    return blk, blk.arrays()


def test_single_shard_shapes(tmp_path):
    blk, a = _arrays()
    write_safetensors(tmp_path / "model.safetensors", checkpoint_tensors(PREFIX, a))
    dt, shp = qmoe.safetensors_tensor_info(tmp_path, f"{PREFIX}.switch_mlp.gate_proj.weight")
    assert dt == "U32" and shp == (16, 64, 256 * 4 // 32)
    dt, shp = qmoe.safetensors_tensor_info(tmp_path, f"{PREFIX}.switch_mlp.down_proj.scales")
    assert dt == "BF16" and shp == (16, 256, 64 // 64)
    dt, shp = qmoe.safetensors_tensor_info(tmp_path, f"{PREFIX}.shared_expert_gate.weight")
    assert dt == "U32" and shp == (1, 256 * 8 // 32)
    with pytest.raises(KeyError):
        qmoe.safetensors_tensor_info(tmp_path, f"{PREFIX}.no_such_tensor.weight")


def test_sharded_checkpoint(tmp_path):
    blk, a = _arrays()
    t = checkpoint_tensors(PREFIX, a)
    names = sorted(t)
    write_safetensors(tmp_path / "model-00001-of-00002.safetensors", {n: t[n] for n in names[::2]})
    write_safetensors(tmp_path / "model-00002-of-00002.safetensors", {n: t[n] for n in names[1::2]})
    for n in names:
        dt, shp = qmoe.safetensors_tensor_info(tmp_path, n)
        assert dt == t[n][0] and shp == tuple(t[n][1].shape)


def test_malformed_headers_are_refused(tmp_path):
    (tmp_path / "a.safetensors").write_bytes((1 << 40).to_bytes(8, "little") + b"{}")
    with pytest.raises(KeyError):
        qmoe.safetensors_tensor_info(tmp_path, "x")
    bad = tmp_path / "b"
    bad.mkdir()
    hdr = b'{"x": {"dtype": "U32", "shape": [4], "data_offsets": [0, 8]}}'   # 4 x U32 needs 16 bytes
    (bad / "m.safetensors").write_bytes(len(hdr).to_bytes(8, "little") + hdr + bytes(8))
    with pytest.raises(KeyError):
        qmoe.safetensors_tensor_info(bad, "x")
    empty = tmp_path / "c"
    empty.mkdir()
    with pytest.raises(KeyError):
        qmoe.safetensors_tensor_info(empty, "x")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_open_refused_without_gpu(tmp_path):
    blk, a = _arrays()
    write_safetensors(tmp_path / "model.safetensors", checkpoint_tensors(PREFIX, a))
    with pytest.raises(qmoe.EngineError):
        qmoe.MoeBlock.from_safetensors(tmp_path, PREFIX, top_k=4)
