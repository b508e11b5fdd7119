"""CPU: the MLX safetensors reader and the config / weight loader.

A model directory is written in the published safetensors layout from seeded MLX-layout
weights (one file or several with an index, flat or ".inner" names), read back through the
library's reader, and compared byte for byte -- whole tensors and every tensor-parallel
rank's slice (the slices shard_weights takes)."""
import numpy as np
import pytest

from oracle.model_ref import synth_weights_numpy
from tests.mlx_checkpoint import write_model_dir


def _args():
    from higgs_b200.model import tiny_args
    return tiny_args("qwen3", layers=2)


@pytest.mark.parametrize("shards,inner", [(1, False), (3, False), (2, True)])
def test_reader_roundtrip_and_names(tmp_path, shards, inner):
    from higgs_b200.loader import SafetensorsDir, load_model_args
    args = _args()
    w = synth_weights_numpy(args, seed=0)
    write_model_dir(str(tmp_path), args, w, shards=shards, inner_names=inner)
    assert load_model_args(str(tmp_path)) == args
    with SafetensorsDir(str(tmp_path)) as st:
        assert sorted(st.names()) == sorted(w)
        for name, a in w.items():
            i = st.find(name)
            assert i >= 0, name
            got = st.read_host(i)
            assert np.array_equal(got.reshape(a.shape), a), name
        assert st.find("model.layers.0.self_attn.q_proj.inner.weight") >= 0  # either naming
        assert st.find("no.such.tensor") == -1


@pytest.mark.parametrize("model_type,world", [("qwen3", 2), ("qwen3", 4), ("qwen3_moe", 2)])
def test_shard_slices_equal_shard_weights(tmp_path, model_type, world):
    """Every rank's slice read from the file equals shard_weights' slice of the same tensor."""
    import dataclasses

    from higgs_b200.loader import SafetensorsDir
    from higgs_b200.model import shard_plan, shard_weights, tiny_args
    from tests.test_tp_cpu import tp_args
    if model_type == "qwen3_moe":
        args = dataclasses.replace(tiny_args(model_type, layers=2), intermediate_size=1024)
    else:
        args = tp_args()
    w = synth_weights_numpy(args, seed=1)
    write_model_dir(str(tmp_path), args, w, shards=2)
    with SafetensorsDir(str(tmp_path)) as st:
        for rank in range(world):
            ref = shard_weights(args, w, rank, world)
            for name, a in w.items():
                rows = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
                r0, nr, c0, nc = shard_plan(args, name, rows, a.shape[-1], rank, world)
                got = st.read_host(st.find(name), r0, nr, c0, nc)
                assert np.array_equal(got.reshape(-1), np.ascontiguousarray(ref[name]).reshape(-1)), (name, rank)


def test_reader_rejects_bad_files(tmp_path):
    from higgs_b200 import ffi
    from higgs_b200.loader import SafetensorsDir, load_model_args
    with pytest.raises(ffi.HiggsError, match="no safetensors files"):
        SafetensorsDir(str(tmp_path))
    (tmp_path / "model.safetensors").write_bytes((1 << 40).to_bytes(8, "little") + b"{}")
    with pytest.raises(ffi.HiggsError, match="header length"):
        SafetensorsDir(str(tmp_path))
    hdr = b'{"a": {"dtype": "U32", "shape": [4], "data_offsets": [0, 8]}}'
    (tmp_path / "model.safetensors").write_bytes(len(hdr).to_bytes(8, "little") + hdr + b"\0" * 16)
    with pytest.raises(ffi.HiggsError, match="data offsets"):
        SafetensorsDir(str(tmp_path))
    hdr = b'{"a": {"dtype": "U32", "shape": [2, 2], "data_offsets": [0, 16]}}'
    (tmp_path / "model.safetensors").write_bytes(len(hdr).to_bytes(8, "little") + hdr + bytes(range(16)))
    with SafetensorsDir(str(tmp_path)) as st:
        with pytest.raises(ffi.HiggsError, match="slice outside"):
            st.read_host(0, 1, 2, 0, 2)
        assert st.read_host(0, 1, 1, 1, 1).view(np.uint8).reshape(-1).tolist() == [12, 13, 14, 15]
    (tmp_path / "config.json").write_text('{"model_type": "qwen3", "quantization": {"group_size": 32, "bits": 4}}')
    with pytest.raises(ValueError, match="group-64"):
        load_model_args(str(tmp_path))
