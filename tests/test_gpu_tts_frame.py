"""A whole TTS decode frame on the device against the oracle, teacher-forced.

runner.TtsFrame runs run_decode_loop's per-frame work (src/tts_native.c:1042-1165: talker
step, cb0 suppression + repetition penalty + top-k, the code predictor's 15 sub-codes, the
codec_sum feedback) as library calls. The oracle replays each frame from the same weights and
the GPU's own sampled tokens: every logits vector the GPU sampled from must match the oracle's
(max |d| / max(1, |ref|) <= 1e-4 after up to 2 + 2 stacked layers per row) and every token
must be the one the reference's tts_sample_topk picks from those logits with the same draw
(skipped only when the draw falls within rounding of a cumulative boundary).
"""
import numpy as np
import pytest

import oracle
import runner
from conftest import max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CFG = runner.TtsConfig(name="tiny", hidden=256, inter=384, layers=2, cp_inter=384, cp_layers=2,
                       max_seq=64)
TOL = 1e-4


def np32(t):
    return t.detach().float().cpu().numpy()


def bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


class OracleFrame:
    """The same frame restated with the oracle's CPU functions, fed the GPU's tokens."""

    def __init__(self, tf):
        c = self.c = tf.cfg
        self.tf = tf
        L = lambda ls: [{k: (bits(v) if v.dtype == torch.bfloat16 else np32(v))  # noqa: E731
                         for k, v in d.items()} for d in ls]
        self.talker, self.cp = L(tf.talker), L(tf.cp)
        self.final_norm, self.cp_norm = np32(tf.final_norm), np32(tf.cp_norm)
        self.codec_head, self.codec_embed = bits(tf.codec_head), bits(tf.codec_embed)
        self.cp_heads = [bits(h) for h in tf.cp_heads]
        self.cp_embed = [bits(e) for e in tf.cp_embed]
        self.cos, self.sin = np32(tf.cos), np32(tf.sin)
        self.trailing, self.draws = np32(tf.trailing), np32(tf.draws)
        kvd = c.n_kv * c.head_dim
        self.kc = np.zeros((c.layers, 1, c.max_seq, kvd), np.float32)
        self.vc = np.zeros_like(self.kc)
        self.cp_kc = np.zeros((c.cp_layers, 1, c.groups, kvd), np.float32)
        self.cp_vc = np.zeros_like(self.cp_kc)
        self.codec_sum = np32(tf.codec_sum).copy()  # the initial input, before any frame
        self.hist = []
        self.pos = 0

    def layers(self, x, layers, kc, vc, pos, inter):
        c = self.c
        qd, kvd = c.n_q * c.head_dim, c.n_kv * c.head_dim
        for i, L in enumerate(layers):
            qkv = oracle.linear_bf16(oracle.rms_norm(x, L["in_norm"], c.eps), L["wqkv"])
            q, k = oracle.qk_norm_rope(qkv[:, :qd], qkv[:, qd:qd + kvd], L["q_norm"], L["k_norm"],
                                       self.cos, self.sin, np.array([pos], np.int32), c.n_q,
                                       c.n_kv, c.head_dim, c.eps, bf16=False)
            kc[i, 0, pos], vc[i, 0, pos] = k[0], qkv[0, qd + kvd:]
            attn = oracle.decode_attention(q, kc[i], vc[i], np.array([pos], np.int32), c.n_q,
                                           c.n_kv, c.head_dim)
            x = oracle.add_inplace(x, oracle.linear_bf16(attn, L["wo"]))
            gu = oracle.linear_bf16(oracle.rms_norm(x, L["post_norm"], c.eps), L["wgu"])
            x = oracle.add_inplace(x, oracle.linear_bf16(oracle.swiglu_multiply(gu, inter),
                                                         L["wd"]))
        return x

    def check_sample(self, logits_gpu, token, u, history):
        c = self.c
        lg = oracle.repetition_penalty(logits_gpu, np.array(history, np.int32), c.penalty) \
            if history is not None else logits_gpu
        tok, margin, total = oracle.sample_topk(lg, c.temperature, c.top_k, u)
        if margin > 1e-6 * total:
            assert tok == token, (tok, token)

    def frame(self, f, codes, recorded):
        c = self.c
        x = self.layers(self.codec_sum, self.talker, self.kc, self.vc, self.pos, c.inter)
        hidden = oracle.rms_norm(x, self.final_norm, c.eps)
        logits = oracle.linear_bf16(hidden, self.codec_head)
        keep = logits[0, c.eos]
        logits[0, c.suppress_start:] = -1.0e9
        logits[0, c.eos] = keep
        got = recorded.pop(0)
        assert max_rel_err(got, logits) <= TOL
        cb0 = int(codes[f, 0])
        self.check_sample(got[0], cb0, self.draws[f, 0], self.hist)
        self.hist.append(cb0)
        self.layers(hidden, self.cp, self.cp_kc, self.cp_vc, 0, c.cp_inter)
        emb = oracle.gather_bf16_to_f32(self.codec_embed, np.array([cb0], np.int32))
        self.codec_sum = emb.copy()
        for j in range(c.groups - 1):
            y = self.layers(emb, self.cp, self.cp_kc, self.cp_vc, j + 1, c.cp_inter)
            lg = oracle.linear_bf16(oracle.rms_norm(y, self.cp_norm, c.eps), self.cp_heads[j])
            got = recorded.pop(0)
            assert max_rel_err(got, lg) <= TOL, (f, j)
            sub = int(codes[f, j + 1])
            self.check_sample(got[0], sub, self.draws[f, j + 1], None)
            emb = oracle.gather_bf16_to_f32(self.cp_embed[j], np.array([sub], np.int32))
            self.codec_sum = oracle.add_inplace(self.codec_sum, emb)
        self.codec_sum = oracle.add_inplace(self.codec_sum, self.trailing[f:f + 1])
        self.pos += 1


def test_frames_match_oracle_teacher_forced():
    frames = 3
    tf = runner.TtsFrame(CFG, frames, seed=5)
    ora = OracleFrame(tf)  # snapshot of the initial state before any frame runs
    tf.record = []
    for _ in range(frames):
        tf.frame()
    torch.cuda.synchronize()
    assert int(tf.err.item()) == 0
    codes = tf.codes.cpu().numpy()
    recorded = [np32(r) for r in tf.record]
    assert len(recorded) == frames * CFG.groups
    assert ((codes[:, 1:] >= 0) & (codes[:, 1:] < CFG.codec_vocab)).all()
    assert ((codes[:, 0] >= 0) & (codes[:, 0] < CFG.talker_vocab)).all()
    for f in range(frames):
        ora.frame(f, codes, recorded)
    # the device history holds the cb0 of every frame
    assert tf.history.cpu().numpy()[0, :frames].tolist() == codes[:, 0].tolist()
    assert int(tf.hist_len.item()) == frames


def test_graph_replay_equals_direct_launches():
    # the same frames as one captured CUDA graph replayed per frame: identical codes and state
    frames = 3
    a, b = runner.TtsFrame(CFG, frames, seed=9), runner.TtsFrame(CFG, frames, seed=9)
    for _ in range(frames):
        a.frame()
        b.frame(graph=True)
    torch.cuda.synchronize()
    assert torch.equal(a.codes, b.codes)
    assert torch.equal(a.codec_sum, b.codec_sum)
    assert int(a.pos.item()) == int(b.pos.item()) == frames


def test_masked_range_and_history_append():
    import lai
    lg = torch.randn(2, 3072, device="cuda")
    ref = lg.clone()
    lai.logits_mask_range(lg, 2048, 3072, keep=2150)
    ref[:, 2048:] = -1.0e9
    ref[:, 2150] = lg[:, 2150]
    assert torch.equal(lg, ref)
    hist = torch.zeros((2, 3), dtype=torch.int32, device="cuda")
    n = torch.tensor([0, 2], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for t in (7, 9):
        lai.history_append(hist, n, torch.tensor([t, t + 1], dtype=torch.int32, device="cuda"),
                           err=err)
    assert hist.cpu().tolist() == [[7, 9, 0], [0, 0, 8]]
    assert n.cpu().tolist() == [2, 3]
    assert int(err.item()) == lai.LAI_DEVERR_POSITION  # row 1 was full on the second append
