"""On-disk format of packed weights (packed_io) and decoders loaded from it."""

from __future__ import annotations

import pytest
import torch

from dequant_project_b200.decoder import DecoderConfig, PackedModel, TPDecoder
from dequant_project_b200.packed_io import load_packed, save_packed
from dequant_project_b200.packer import QuantConfig, dequantize, quantize_tensor

FORMATS = [QuantConfig(4, 128, False), QuantConfig(4, 128, True, "interleaved"),
           QuantConfig(2, 64, False), QuantConfig(8, None, True), QuantConfig(8, None, False)]


def test_round_trip_every_format(tmp_path):
    torch.manual_seed(0)
    packed = {f"w{i}": quantize_tensor(torch.randn(48, 512, dtype=torch.float16) * 0.02, c)
              for i, c in enumerate(FORMATS)}
    emb = torch.randn(10, 512, dtype=torch.float16)
    save_packed(tmp_path / "m.pt", packed, {"embed": emb}, meta={"note": "x"})
    back, tensors, meta = load_packed(tmp_path / "m.pt")
    assert meta == {"note": "x"} and torch.equal(tensors["embed"], emb)
    assert set(back) == set(packed)
    for k, pw in packed.items():
        b = back[k]
        assert b.config == pw.config and tuple(b.shape) == tuple(pw.shape)
        assert torch.equal(b.qweight, pw.qweight) and torch.equal(b.scales, pw.scales)
        assert (b.zeros is None) == (pw.zeros is None)
        assert pw.zeros is None or torch.equal(b.zeros, pw.zeros)
        assert torch.equal(dequantize(b), dequantize(pw))


def test_rejects_other_files_and_bad_records(tmp_path):
    torch.save({"a": torch.zeros(3)}, tmp_path / "other.pt")
    with pytest.raises(ValueError, match="not a"):
        load_packed(tmp_path / "other.pt")
    pw = quantize_tensor(torch.randn(16, 256, dtype=torch.float16), FORMATS[0])
    save_packed(tmp_path / "ok.pt", {"w": pw})
    blob = torch.load(tmp_path / "ok.pt", weights_only=True)
    blob["packed"]["w"]["shape"] = [16, 512]          # words no longer match K
    torch.save(blob, tmp_path / "bad.pt")
    with pytest.raises(ValueError, match="qweight must be int32"):
        load_packed(tmp_path / "bad.pt")


def cpu_linear(x, pw):
    return (x.float() @ dequantize(pw).float().t()).to(torch.float16)


@pytest.mark.parametrize("quantize_head", (True, False))
def test_decoder_from_file_matches_seeded_decoder(tmp_path, quantize_head):
    cfg = DecoderConfig(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, intermediate=640,
                        vocab=1000)
    q = QuantConfig(4, 64, False)
    PackedModel.build(cfg, q, seed=3, quantize_lm_head=quantize_head).save(tmp_path / "d.pt")
    loaded = PackedModel.load(tmp_path / "d.pt")
    assert loaded.cfg == cfg and loaded.qcfg == q
    a = TPDecoder(cfg, q, seed=3, batch=2, kv_len=16, quantize_lm_head=quantize_head,
                  linear_fn=cpu_linear)
    b = TPDecoder(cfg, q, seed=3, batch=2, kv_len=16, weights=loaded, linear_fn=cpu_linear)
    tok = torch.tensor([1, 999])
    assert torch.equal(a.step(tok, 16), b.step(tok, 16))
    with pytest.raises(ValueError, match="differs"):
        TPDecoder(cfg, QuantConfig(2, 64, False), weights=loaded, linear_fn=cpu_linear)


def test_decode_bench_loads_a_saved_model(tmp_path):
    """decode_bench's --save-weights / --weights source (CPU tensors here)."""
    from dequant_project_b200 import decode_bench
    cfg = DecoderConfig(n_layers=1, hidden=256, n_heads=4, n_kv_heads=2, intermediate=640,
                        vocab=500)
    q = QuantConfig(2, 64, False)
    PackedModel.build(cfg, q, seed=4).save(tmp_path / "m.pt")
    got_cfg, got_q, model = decode_bench.model_source(
        decode_bench.default_args(weights=str(tmp_path / "m.pt")), torch.device("cpu"))
    assert got_cfg == cfg and got_q == q and isinstance(model, PackedModel)
    cfg7, q7, none = decode_bench.model_source(decode_bench.default_args(layers=2),
                                               torch.device("cpu"))
    assert none is None and cfg7.n_layers == 2 and cfg7.hidden == 4096 and q7.bits == 4
