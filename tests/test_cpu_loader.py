"""Checkpoint reading on the CPU: the three safetensors layouts of
loader.py:75-114, name mapping (with and without a ``model.`` prefix), config
parsing and the config round trip.  Quantisation and device upload are in
test_gpu_loader.py."""
import importlib

import pytest
import torch

from helpers import tiny_cfg
from loader_util import make_checkpoint


@pytest.fixture(scope="module")
def L(pkg):
    return importlib.import_module("mirror-sd_b200.loader")


@pytest.mark.parametrize("layout,prefix", [("single", ""), ("sharded", ""), ("glob", "model.")])
def test_read_layouts(L, tmp_path, layout, prefix):
    ocfg = tiny_cfg()
    want = make_checkpoint(tmp_path, ocfg, seed=1, layout=layout, prefix=prefix)
    files = L.weight_files(tmp_path)
    assert len(files) == (1 if layout == "single" else 2)
    got = L.read_tensors(tmp_path)
    assert set(got) == set(want)
    for k, v in want.items():
        assert got[k].dtype == torch.bfloat16
        assert torch.equal(got[k].float(), v), k


def test_config_and_round_trip(L, pkg, tmp_path):
    ocfg = tiny_cfg()
    make_checkpoint(tmp_path, ocfg)
    cfg = L.load_config(tmp_path)
    assert (cfg.hidden_size, cfg.num_hidden_layers, cfg.intermediate_size) == (256, 2, 256)
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.block_size) == (4, 2, 8)
    assert cfg.target_layer_ids == [0, 1, 2, 3, 4]
    back = pkg.DFlashConfig.from_dict(cfg.to_dict())
    assert back == cfg
    cfg2 = L.load_config(tmp_path, {"rope_theta": 5.0e5})
    assert cfg2.rope_theta == 5.0e5


def test_missing_tensor_and_bad_shape(L, tmp_path):
    ocfg = tiny_cfg()
    make_checkpoint(tmp_path, ocfg)
    cfg = L.load_config(tmp_path)
    cfg.hidden_size = 512   # fc.weight no longer matches
    with pytest.raises(ValueError):
        L.load_dflash_weights(tmp_path, cfg, device="cpu")
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(FileNotFoundError):
        L.weight_files(empty)
