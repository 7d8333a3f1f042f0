"""Device repetition penalty + top-k sampling against the reference's sampling code.

tts_apply_repetition_penalty / tts_sample_topk (src/tts_sampling.c:19-109). The draw the
reference takes from libc rand() is passed in as u. Penalised logits must match
bit for bit. Tokens must be identical, except where r = u * sum lies within 1e-6 * sum of a
cumulative boundary: CUDA's expf and glibc's may differ in the last bit of each term, which
moves a running sum by about 6e-8 * sum, so there the draw is counted (and must stay rare:
about 2 * top_k * 1e-6 of the draws) rather than compared.
"""
import numpy as np
import pytest

import lai
import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"


def batch(rows, vocab, seed, hist=64):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((rows, vocab)) * rng.uniform(0.5, 4, (rows, 1))).astype(np.float32)
    logits[::5, rng.integers(0, vocab, 8)] = logits[::5].max()  # ties at the top in some rows
    history = rng.integers(-3, vocab + 3, (rows, hist)).astype(np.int32)
    hist_len = rng.integers(0, hist + 1, rows).astype(np.int32)
    u = rng.uniform(0, 1, rows).astype(np.float32)
    return logits, history, hist_len, u


def run(logits, history, hist_len, u, penalty, temperature, top_k):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    lg = t(logits)
    tok = lai.sample_topk(lg, t(u), temperature, top_k, t(history), t(hist_len), penalty)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), lg.cpu().numpy()


@pytest.mark.parametrize("vocab,top_k,temp,penalty", [(3072, 50, 0.9, 1.05), (2048, 50, 0.7, 1.0),
                                                      (3072, 1, 1.0, 1.3), (300, 0, 1.3, 1.1),
                                                      (3072, 3072, 0.8, 1.0), (100, 7, 0.5, 2.0),
                                                      (3072, 600, 1.0, 1.05)])
def test_sample_topk_matches_oracle(vocab, top_k, temp, penalty):
    rows = 256
    logits, history, hist_len, u = batch(rows, vocab, vocab + top_k)
    tok, lg = run(logits, history, hist_len, u, penalty, temp, top_k)
    ambiguous = 0
    for r in range(rows):
        pen = oracle.repetition_penalty(logits[r], history[r, :hist_len[r]], penalty)
        assert np.array_equal(lg[r], pen), r
        want, margin, s = oracle.sample_topk(pen, temp, top_k, u[r])
        if margin <= 1e-6 * s:
            ambiguous += 1
            continue
        assert tok[r] == want, (r, tok[r], want)
    assert ambiguous <= rows // 50


@pytest.mark.skipif(not oracle.have_ref_sampling(), reason="reference sampling not built")
def test_sample_topk_matches_reference_build():
    # the reference's own compiled tts_sample_topk, rand() driven by srand(seed)
    rows, vocab, top_k, temp = 128, 3072, 50, 0.9
    logits, _, _, _ = batch(rows, vocab, 77)
    seeds = list(range(5000, 5000 + rows))
    u = np.array([oracle.ref_rand_draw(sd) for sd in seeds], np.float32)
    tok, _ = run(logits, np.zeros((rows, 1), np.int32), np.zeros(rows, np.int32), u, 1.0, temp,
                 top_k)
    same = sum(int(tok[r] == oracle.ref_sample_topk(logits[r], temp, top_k, seeds[r]))
               for r in range(rows))
    assert same >= rows - 2  # the odd expf-at-a-boundary draw (see module docstring)


def test_sample_topk_argument_checks():
    L = lai.load()
    import ctypes
    from conftest import arena_ptr
    P = arena_ptr(1 << 20)  # real memory: a regressed check would still stay in bounds
    f = L.lai_sample_topk_f32
    assert f(P, P, 0, 1, None, None, 0, 1.0, 1.0, 5, P, None) == lai.LAI_ERR_INVALID
    assert f(P, P, 100, 1, P, None, 4, 1.0, 1.0, 5, P, None) == lai.LAI_ERR_INVALID
    assert f(P, P, 1 << 22, 1, None, None, 0, 1.0, 1.0, 1 << 20, P, None) == lai.LAI_ERR_TOOBIG
    assert f(P, P, 100, 0, None, None, 0, 1.0, 1.0, 5, P, None) == lai.LAI_OK
