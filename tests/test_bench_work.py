"""The algorithmic work bench.py reports throughput against, recomputed from the model's layer
shapes (the weight manifest): text-side FLOPs per token, and the config-3 input generator."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("kk_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _lin(m, name):
    out_f, in_f = m[name][0][:2]
    return 2 * out_f * in_f


def test_text_side_flops_per_token_match_the_layer_shapes(kk):
    m = kk.weights.manifest()
    L = "bert.encoder.albert_layer_groups.0.albert_layers.0."
    albert = _lin(m, "bert.encoder.embedding_hidden_mapping_in.weight") + 12 * sum(
        _lin(m, L + n) for n in ("attention.query.weight", "attention.key.weight", "attention.value.weight",
                                 "attention.dense.weight", "ffn.weight", "ffn_output.weight"))

    def bilstm(p):
        return 2 * (_lin(m, p + "weight_ih_l0") + _lin(m, p + "weight_hh_l0"))

    cout, cin, k = m["text_encoder.cnn.0.0.weight_v"][0]
    text_enc = 3 * 2 * cout * cin * k + bilstm("text_encoder.lstm.")
    dur = (_lin(m, "bert_encoder.weight") + sum(bilstm(f"predictor.text_encoder.lstms.{i}.") for i in (0, 2, 4))
           + bilstm("predictor.lstm.") + _lin(m, "predictor.duration_proj.linear_layer.weight"))
    b = _bench()
    assert abs(albert - 132.3e6) / 132.3e6 < 1e-3
    assert abs(text_enc - 11.0e6) / 11.0e6 < 2e-3
    assert abs(dur - 15.5e6) / 15.5e6 < 2e-3
    assert abs((albert + text_enc + dur) - b.TEXT_FLOP_PER_TOKEN) / b.TEXT_FLOP_PER_TOKEN < 1e-3
    # attention: QK^T and PV over the sequence, 12 layers of hidden 768
    assert b.ATTN_FLOP_PER_TOKEN_PER_T == 12 * 2 * 2 * 768


def test_config3_inputs():
    b = _bench()
    toks, style = b.config3_lines(3000)
    lens = np.array([len(t) for t in toks])
    assert len(toks) == 256 and lens.min() >= 16 and lens.max() <= 510
    assert all(t.min() >= 1 and t.max() <= 177 for t in toks)
    assert style.shape == (256,)
    toks2, _ = b.config3_lines(3000)
    assert all(np.array_equal(a, c) for a, c in zip(toks, toks2))
