"""Weight I/O compatibility with the reference (src/sisa/checkpoint.py; its tests/test_checkpoint.py is the
model for these cases). Pinned by tests/golden/ckpt_case.pt: files written by the reference's own
save_pretrained, its logits, and its key conversion."""
from __future__ import annotations

import json
import pickle

import pytest
import torch

import sisa_b200 as sisa
from sisa_b200.checkpoint import convert_state_dict, infer_config_from_state_dict, load_paper_checkpoint

from golden.make_golden import paper_layout


def tiny(seed=0, **over):
    cfg = dict(vocab_size=257, d_model=64, n_layer=2, n_head=2, d_ff=96, d_state=8, attn_impl="torch")
    cfg.update(over)
    torch.manual_seed(seed)
    model = sisa.SISAForCausalLM(sisa.SISAConfig(**cfg))
    with torch.no_grad():   # W_C = 0 at init would hide the SSM term
        for layer in model.layers:
            layer.attn.W_C.weight.normal_(0.0, 0.1)
    return model.eval()


def ids(seq_len=20):
    return torch.randint(0, 257, (2, seq_len), generator=torch.Generator().manual_seed(0))


class _Opaque:
    """A pickled object that ``torch.load(weights_only=True)`` refuses."""

    d_ff = 2048


def _write_ref_dir(case, tmp_path, names):
    tmp_path.mkdir(parents=True, exist_ok=True)
    for name in names:
        (tmp_path / name).write_bytes(case["files"][name])
    return tmp_path


@pytest.mark.parametrize("weights", ["model.safetensors", "pytorch_model.bin"])
def test_loads_directory_written_by_reference(golden, tmp_path, weights):
    case = golden("ckpt_case")
    d = _write_ref_dir(case, tmp_path, ["config.json", weights])
    model = sisa.SISAForCausalLM.from_pretrained(d)
    assert not model.training and model.config.attn_impl == "torch"
    assert list(model.state_dict().keys()) == case["state_dict_keys"]
    with torch.no_grad():
        logits = model(case["ids"]).logits
    torch.testing.assert_close(logits, case["logits"], rtol=1e-5, atol=1e-5)


def test_written_directory_matches_reference_format(golden, tmp_path):
    case = golden("ckpt_case")
    src = sisa.SISAForCausalLM.from_pretrained(_write_ref_dir(case, tmp_path / "ref", ["config.json",
                                                                                     "model.safetensors"]))
    src.save_pretrained(tmp_path / "ours")
    assert json.loads((tmp_path / "ours" / "config.json").read_text()) == json.loads(case["files"]["config.json"])
    from safetensors import safe_open

    for name in ("ours", "ref"):
        with safe_open(str(tmp_path / name / "model.safetensors"), "pt") as f:
            assert f.metadata() == {"format": "pt"}
            keys = sorted(f.keys())
            if name == "ours":
                ours = {k: f.get_tensor(k) for k in keys}
            else:
                theirs = {k: f.get_tensor(k) for k in keys}
    assert ours.keys() == theirs.keys()
    for k in ours:
        assert ours[k].dtype == theirs[k].dtype and torch.equal(ours[k], theirs[k]), k


def test_key_conversion_matches_reference(golden):
    case = golden("ckpt_case")
    for src, want in case["key_map"].items():
        assert next(iter(convert_state_dict({src: torch.zeros(1)}))) == want, src
    from safetensors.torch import load as load_safetensors

    weights = load_safetensors(case["files"]["model.safetensors"])
    assert set(convert_state_dict(paper_layout(weights))) == set(case["state_dict_keys"])
    assert infer_config_from_state_dict(paper_layout(weights, "module.")).to_dict() == case["inferred"]


@pytest.mark.parametrize("prefix", ["", "module.", "_orig_mod.", "module._orig_mod."])
def test_paper_layout_round_trip(prefix):
    src = tiny(seed=1)
    converted = convert_state_dict(paper_layout(src.state_dict(), prefix))
    assert set(converted) == set(src.state_dict())
    assert list(convert_state_dict(converted)) == list(converted)                 # idempotent
    dst = sisa.SISAForCausalLM(infer_config_from_state_dict(converted, attn_impl="torch")).eval()
    dst.load_state_dict(converted, strict=True)
    with torch.no_grad():
        assert torch.equal(dst(ids()).logits, src(ids()).logits)


def test_colliding_keys_raise():
    with pytest.raises(ValueError, match="map to"):
        convert_state_dict({"layers.0.W_Q.weight": torch.zeros(1), "layers.0.attn.W_Q.weight": torch.zeros(1)})


def test_infer_config_reads_shapes_only():
    src = tiny(seed=2, d_ff=200, n_layer=3)
    cfg = infer_config_from_state_dict(paper_layout(src.state_dict()))
    for field in ("vocab_size", "d_model", "n_layer", "n_head", "d_ff", "d_state"):
        assert getattr(cfg, field) == getattr(src.config, field), field
    with pytest.raises(ValueError, match="cannot be overridden"):
        infer_config_from_state_dict(paper_layout(src.state_dict()), d_ff=100)
    with pytest.raises(ValueError, match="not a SISA state dict"):
        infer_config_from_state_dict({"embed.weight": torch.zeros(3, 4)})
    sd = {k.replace("layers.1.", "layers.5."): v for k, v in paper_layout(src.state_dict()).items()}
    with pytest.raises(ValueError, match="not contiguous"):
        infer_config_from_state_dict(sd)


def test_load_paper_checkpoint_drops_training_state(tmp_path):
    src = tiny(seed=3)
    path = tmp_path / "final.pt"
    torch.save({"model": paper_layout(src.state_dict()), "optimizer": {"state": {}, "param_groups": []},
                "scheduler": {"last_epoch": 7}, "step": 7,
                "config": {"d_ff": 2048, "data_dir": "/data/tokens", "run_name": "x"}}, path)
    model = load_paper_checkpoint(path, attn_impl="torch")
    assert not model.training and model.config.d_ff == src.config.d_ff
    assert model.num_parameters() == src.num_parameters()
    with torch.no_grad():
        assert torch.equal(model(ids()).logits, src(ids()).logits)
    assert not [v for v in vars(model).values() if isinstance(v, dict) and "data_dir" in v]
    half = load_paper_checkpoint(path, dtype=torch.bfloat16)
    assert half.embed.weight.dtype == torch.bfloat16
    assert half.layers[0].attn.lambda_raw.dtype == torch.float32


def test_plain_state_dict_file(tmp_path):
    src = tiny(seed=4)
    torch.save(paper_layout(src.state_dict()), tmp_path / "w.pt")
    model = load_paper_checkpoint(tmp_path / "w.pt", attn_impl="torch")
    with torch.no_grad():
        assert torch.equal(model(ids()).logits, src(ids()).logits)


def test_pickled_objects_need_trust(tmp_path):
    src = tiny(seed=5)
    path = tmp_path / "final.pt"
    torch.save({"model": paper_layout(src.state_dict()), "config": _Opaque()}, path)
    with pytest.raises(pickle.UnpicklingError, match="trust_pickle"):
        load_paper_checkpoint(path)
    model = load_paper_checkpoint(path, trust_pickle=True, attn_impl="torch")
    with torch.no_grad():
        assert torch.equal(model(ids()).logits, src(ids()).logits)


def test_key_and_shape_mismatches_raise(tmp_path):
    src = tiny(seed=6)
    sd = paper_layout(src.state_dict())
    del sd["layers.1.forget_proj.bias"]
    torch.save({"model": sd}, tmp_path / "a.pt")
    with pytest.raises(ValueError, match="missing"):
        load_paper_checkpoint(tmp_path / "a.pt")
    sd = paper_layout(src.state_dict())
    sd["layers.0.extra.weight"] = torch.zeros(1)
    torch.save({"model": sd}, tmp_path / "b.pt")
    with pytest.raises(ValueError, match="unexpected"):
        load_paper_checkpoint(tmp_path / "b.pt")
    sd = paper_layout(src.state_dict())
    sd["layers.1.ffn._orig_mod.w_up.weight"] = torch.zeros(10, 64)
    torch.save({"model": sd}, tmp_path / "c.pt")
    with pytest.raises(ValueError, match="shape mismatch"):
        load_paper_checkpoint(tmp_path / "c.pt")
    torch.save({"something": 1}, tmp_path / "d.pt")
    with pytest.raises(ValueError, match="state dict"):
        load_paper_checkpoint(tmp_path / "d.pt")


@pytest.mark.parametrize("safe", [True, False])
def test_save_and_from_pretrained(tmp_path, safe):
    src = tiny(seed=7)
    src.save_pretrained(tmp_path, safe_serialization=safe)
    assert (tmp_path / "config.json").exists()
    assert (tmp_path / ("model.safetensors" if safe else "pytorch_model.bin")).exists()
    loaded = sisa.SISAForCausalLM.from_pretrained(tmp_path)
    assert loaded.config == src.config and not loaded.training
    with torch.no_grad():
        assert torch.equal(loaded(ids()).logits, src(ids()).logits)
    other = sisa.SISAForCausalLM.from_pretrained(tmp_path, attn_impl="auto", dtype=torch.bfloat16)
    assert other.config.attn_impl == "auto" and other.embed.weight.dtype == torch.bfloat16


def test_save_removes_stale_weights(tmp_path):
    src = tiny(seed=8)
    src.save_pretrained(tmp_path, safe_serialization=False)
    src.save_pretrained(tmp_path, safe_serialization=True)
    assert not (tmp_path / "pytorch_model.bin").exists() and (tmp_path / "model.safetensors").exists()
    src.save_pretrained(tmp_path, safe_serialization=False)
    assert (tmp_path / "pytorch_model.bin").exists() and not (tmp_path / "model.safetensors").exists()


def test_from_pretrained_errors(tmp_path):
    with pytest.raises(ValueError, match="not a directory"):
        sisa.SISAForCausalLM.from_pretrained(tmp_path / "missing")
    tiny().save_pretrained(tmp_path)
    (tmp_path / "model.safetensors").unlink()
    with pytest.raises(FileNotFoundError):
        sisa.SISAForCausalLM.from_pretrained(tmp_path)
