"""Model-shard checkpoints on CPU: a shard saved to safetensors loads into a
shard built from another seed, in place (tensor addresses unchanged, so CUDA
graphs and collective workspaces that hold them stay valid); the TP geometry
names the file, and a file of another model or another key set is refused."""
import pytest
import torch

from kvserve_b200.models.config import get_config
from kvserve_b200.models.llama import LlamaShard


def _shard(seed, tp_rank=1, tp_size=2, name="tiny"):
    return LlamaShard(get_config(name), tp_rank, tp_size, "cpu", seed, max_position=64)


def test_saved_shard_loads_in_place(tmp_path):
    src = _shard(seed=0)
    path = src.save(str(tmp_path / "w"))
    assert path.endswith("w.tp1of2.safetensors")
    dst = _shard(seed=7)
    ptrs = {k: t.data_ptr() for k, t in dst.state_dict().items()}
    assert not torch.equal(dst.layers[0].qkv, src.layers[0].qkv)
    dst.load(str(tmp_path / "w"))
    for k, t in dst.state_dict().items():
        assert torch.equal(t, src.state_dict()[k]), k
        assert t.data_ptr() == ptrs[k], k
    # every layer field and the embedding / head / norm are in the file
    assert len(src.state_dict()) == 3 + 6 * get_config("tiny").num_layers


def test_checkpoint_mismatches_are_refused(tmp_path):
    _shard(seed=0).save(str(tmp_path / "w"))
    with pytest.raises(FileNotFoundError):
        _shard(seed=0, tp_rank=0, tp_size=1).load(str(tmp_path / "w"))     # no file of that geometry
    _shard(seed=0, name="tiny-gqa").save(str(tmp_path / "g"))
    import os
    os.replace(str(tmp_path / "g.tp1of2.safetensors"), str(tmp_path / "x.tp1of2.safetensors"))
    with pytest.raises(ValueError, match="tiny-gqa"):
        _shard(seed=0).load(str(tmp_path / "x"))
    s = _shard(seed=0)
    sd = dict(s.state_dict())
    sd.pop("final_norm")
    with pytest.raises(KeyError, match="final_norm"):
        s.load_state_dict(sd)
    sd = dict(s.state_dict())
    sd["embed"] = sd["embed"][:-1]
    with pytest.raises(ValueError, match="embed"):
        s.load_state_dict(sd)
