"""The encoder's tensors through a synthetic whistle.cact: written with
weights.write_whistle_cact(enc=…) and read back by weights.encoder_weights
(encoder.go:50 LoadInt8's names: encNN.*, enc.mhc_*, enc.final_norm,
stem.*, audio.mel_filters). CQ records come back byte for byte, FP32
records exactly, FP16 records as their float16 rounding; the sizes come
from the audio manifest and the shapes."""

from __future__ import annotations

import numpy as np
import pytest


@pytest.fixture(scope="module")
def written(wb):
    w = wb.synth.DecoderWeights(seed=4510, vocab=8199)
    e = wb.synth.EncoderWeights(seed=5510)
    e.hada_p1, e.hada_p2 = w.hada_p1, w.hada_p2
    return e, wb.weights.write_whistle_cact(w, seed=3, enc=e)


def _same(wb, name, got, want):
    dtype, _ = wb.cact.whistle_storage(name)
    want = np.asarray(want, np.float32).reshape(np.shape(got))
    if dtype == wb.cact.FP16:
        want = want.astype(np.float16).astype(np.float32)
    assert np.array_equal(got, want), name


def test_encoder_round_trip(wb, written):
    e, data = written
    le = wb.weights.load_encoder(data)
    assert (le.n_layers, le.lanes, le.dim, le.heads, le.kv_heads, le.qk, le.vd) == (8, 4, 512, 8, 2, 48, 64)
    assert (le.dw_k, le.na, le.nb, le.rank, le.stem_channels) == (9, 16, 32, 8, 128)
    for l in (0, 5, 7):
        L, W = le.layers[l], e.layers[l]
        for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "pw1", "pw2"):
            assert bytes(L[k].Index) == bytes(W[k].Index) and bytes(L[k].Norms) == bytes(W[k].Norms), (l, k)
        for k in ("pre_hada_0", "norm_in", "conv_out_norm", "q_norm", "dw", "hada_0.w2b", "hada.cond_u"):
            _same(wb, f"enc{l:02d}.{k}", L[k], W[k])
        for k in ("a_pre", "a_res"):
            assert np.float32(L[k]) == np.float16(W[k]).astype(np.float32) or L[k] == np.float32(W[k]), (l, k)
        lo, hi = e.phi_rows("phi_res", l)
        assert le.phi_rows("phi_res", l) == (lo, hi)
    for k in ("phi_pre", "phi_post", "phi_res"):
        assert bytes(getattr(le, k).Index) == bytes(getattr(e, k).Index), k
    for k in ("w", "dw_1", "dw_2"):
        _same(wb, "stem." + k, getattr(le, "stem_" + k), getattr(e, "stem_" + k))
    for k in ("pw_1", "pw_2", "out"):
        assert bytes(getattr(le, "stem_" + k).Index) == bytes(getattr(e, "stem_" + k).Index), k
    _same(wb, "audio.mel_filters", le.mel_filters, e.mel_filters)
    _same(wb, "enc.final_norm", le.final_norm, e.final_norm)
    assert np.array_equal(le.hada_p1, e.hada_p1) and np.array_equal(le.hada_p2, e.hada_p2)


def test_writer_wants_one_permutation_pair(wb):
    w = wb.synth.DecoderWeights(seed=4511, vocab=8199)
    e = wb.synth.EncoderWeights(seed=5511, layers=8)
    with pytest.raises(wb.weights.WeightsError, match="hada_p1/hada_p2 differ"):
        wb.weights.write_whistle_cact(w, enc=e)
