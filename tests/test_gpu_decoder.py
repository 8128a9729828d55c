"""GPU parity of the decoder step (doe_b200.decoder, BASELINE config 5 semantics)
against the numpy restatement oracle/decoder.py on a small model.

Tolerance: the f32 residual stream after all layers within
2e-3 * max(|ref|, 1) (the fp16/bf16 bound); the kernels and the oracle round
at the same points, so what remains is summation order and the odd bf16 / f16
rounding flip that it causes.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import decoder as odec

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from doe_b200 import decoder  # noqa: E402

TOL = 2e-3
SMALL = decoder.DecoderConfig(hidden=512, heads=4, kv_heads=2, ffn=1024, layers=2, batch=8, ctx=100)


def _host_state(dec):
    layers = [{k: v.float().cpu().numpy() for k, v in L.items()} for L in dec.layers]
    caches = [{"k": c.k_pool.cpu().numpy().view(np.uint16).copy(), "v": c.v_pool.cpu().numpy().view(np.uint16).copy(),
               "table": c.block_table.cpu().numpy(), "page_size": c.page_size} for c in dec.caches]
    return layers, caches


def _oracle_step(dec, x0, layers, caches):
    cfg = dec.cfg
    x = x0.copy()
    table = dec.freq_cis.cpu().numpy()
    seq_lens = dec.seq_lens.cpu().numpy()
    for L, c in zip(layers, caches):
        x = odec.layer_partials(x, L, c, qh=dec.qh, kvh=dec.kvh, head_dim=cfg.head_dim, eps=cfg.eps,
                                scale=dec.scale, freq_cis=table, seq_lens=seq_lens, add_residual=True)
    return x


def _x0(cfg, seed=12):
    return np.random.default_rng(seed).standard_normal((cfg.batch, cfg.hidden), dtype=np.float32)


@pytest.mark.parametrize("cfg", [SMALL, decoder.DecoderConfig(hidden=1024, heads=8, kv_heads=1, ffn=2048,
                                                              layers=1, batch=32, ctx=333)])
def test_decoder_step_matches_oracle(cfg):
    dec = decoder.Decoder(cfg, seed=4)
    layers, caches = _host_state(dec)
    x0 = _x0(cfg)
    x = torch.from_numpy(x0).cuda()
    dec.step(x)
    torch.cuda.synchronize()
    assert int(dec.status.item()) == 0
    ref = _oracle_step(dec, x0, layers, caches)
    got = x.cpu().numpy()
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
    assert float(err.max()) <= TOL, f"max rel err {float(err.max()):.3g}"


def test_decoder_graph_replay_equals_eager_step():
    dec = decoder.Decoder(SMALL, seed=5)
    x0 = torch.from_numpy(_x0(SMALL, 3)).cuda()
    x = x0.clone()
    dec.step(x)  # eager warm-up; also the expected result
    torch.cuda.synchronize()
    eager = x.clone()
    x.copy_(x0)
    dec.capture(x)
    x.copy_(x0)
    dec.replay()
    torch.cuda.synchronize()
    assert int(dec.status.item()) == 0
    assert torch.equal(x, eager)
    dec.release()
