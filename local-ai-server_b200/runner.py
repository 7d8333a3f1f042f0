"""Workloads and the row-sharded runner for the per-layer kernels.

A decoder layer's elementwise chain over `tokens` rows (BF16 activations, FP32
norm weights and RoPE table), laid out as the reference's buffers are
(src/tts_native.c:314-338, ensure_prefill_buffers):
    x [T, D] residual, delta_attn / delta_ffn [T, D] (o_proj / down_proj outputs),
    y [T, D] normed, q [T, Hq*hd], k [T, Hkv*hd], gate_up [T, 2I] interleaved,
    act [T, I] SwiGLU output, positions [T] int32, cos/sin [P, hd] FP32.
One step launches, in the reference's per-layer order (src/tts_native.c:553-592):
    add_rmsnorm(x += delta_ffn, y = norm(x; input_norm))   (prev. layer residual fused)
    qk_norm_rope(q, k)
    add_rmsnorm(x += delta_attn, y = norm(x; post_attn_norm))
    swiglu(gate_up -> act)
Rows are independent, so G devices each run their own contiguous row block
(`shard_range`) with no collective; inputs are generated on each device from a
counter-based generator keyed by global element index, so a shard's contents do
not depend on G.
"""
from __future__ import annotations

import dataclasses

import lai

BF16_BYTES = 2


@dataclasses.dataclass(frozen=True)
class LayerConfig:
    name: str
    tokens: int
    dim: int
    inter: int
    n_q: int = 16
    n_kv: int = 8
    head_dim: int = 128
    pos_mode: str = "seq"      # "seq": positions t % pos_period; "random": U[0, pos_period)
    pos_period: int = 1024
    theta: float = 1e6
    eps: float = 1e-6
    vocab: int = 0             # embedding table rows for the gather (0 = no gather)

    # Algorithmic HBM bytes per token per kernel; s = activation element size
    # (2 for BF16 storage, 4 for the FP32 drop-in path).
    def bytes_per_token(self, s: int = BF16_BYTES) -> dict[str, int]:
        return {
            "embed_gather": 2 * self.dim * 2 + 4,                  # BF16 table row, id, output row
            "add_rmsnorm": 4 * self.dim * s,                       # read x, delta; write x', y
            "qk_norm_rope": 2 * (self.n_q + self.n_kv) * self.head_dim * s,  # q, k in place
            "swiglu": 3 * self.inter * s,                          # read 2I, write I
        }

    def kernels(self) -> tuple[str, ...]:
        k = ("add_rmsnorm", "qk_norm_rope", "add_rmsnorm", "swiglu")
        return (("embed_gather",) + k) if self.vocab else k

    def step_bytes_per_token(self, s: int = BF16_BYTES) -> int:
        b = self.bytes_per_token(s)
        return sum(b[k] for k in self.kernels())


# The benchmark configurations C1..C5: ASR-0.6B layer ops (512 tokens), ASR-1.7B layer ops
# (64 x 1024 tokens), TTS-0.6B talker decode (256 rows at random positions), and the
# 2M-token 1.7B chain; C4 (SnakeBeta) is SNAKE_STAGES below.
CONFIGS = {
    "c1": LayerConfig("qwen3-asr-0.6b-decoder-layer", tokens=512, dim=1024, inter=3072,
                      pos_period=512, vocab=151936),
    "c2": LayerConfig("qwen3-asr-1.7b-decoder-layer", tokens=64 * 1024, dim=2048, inter=6144,
                      pos_period=1024),
    "c3": LayerConfig("qwen3-tts-0.6b-talker-decode", tokens=256, dim=1024, inter=3072,
                      pos_mode="random", pos_period=4096, vocab=3072),
    "c5": LayerConfig("qwen3-1.7b-chain-2m", tokens=1 << 21, dim=2048, inter=6144,
                      pos_period=1024),
}

# Decode-step linear path of one layer (fused GEMVs), M tokens per step.
@dataclasses.dataclass(frozen=True)
class DecodeConfig:
    name: str
    dim: int
    inter: int
    q_dim: int = 16 * 128
    kv_dim: int = 8 * 128
    m: int = 1
    layers: int = 28  # talker depth (src/tts_native.h:28): a step streams every layer's weights
    eps: float = 1e-6


DECODE_CONFIGS = {
    "g1": DecodeConfig("qwen3-tts-0.6b-talker-decode-linear", dim=1024, inter=3072),
    "g2": DecodeConfig("qwen3-1.7b-decode-linear", dim=2048, inter=6144),
}

# Vocoder SnakeBeta stages (channels, T) x batch 8 (config 4).
SNAKE_STAGES = [(1536, 2000), (768, 16000), (384, 48000), (192, 96000), (96, 192000)]
SNAKE_BATCH = 8

# Vocoder BigVGAN ResUnits: the four blocks' output widths at the SnakeBeta stages'
# lengths, three units per block with dilations 1, 3, 9 (src/tts_vocoder.c:269, 725-728).
RESUNIT_STAGES = [(768, 16000), (384, 48000), (192, 96000), (96, 192000)]
RESUNIT_BATCH = 8
RESUNIT_DILATIONS = (1, 3, 9)


def resunit_hbm_bytes_per_element(n_units: int, passes: int) -> int:
    """Algorithmic HBM bytes per activation element of lai_voc_resunits_f32: the first
    snake1 reads x and writes s; per unit conv1 reads s and writes h, conv2 reads h and x
    and writes x, and (all but the last unit) the next unit's s. s and h are hi/lo pairs
    (8 bytes) with 3 passes, one TF32 plane (4 bytes) with 1."""
    sp = 8 if passes == 3 else 4
    return (4 + sp) + n_units * (2 * sp + sp + 8) + (n_units - 1) * sp


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced block [start, stop) of n rows for `rank` of `world`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class LayerChain:
    """Device buffers and launches for one shard of a LayerConfig.

    With cfg.vocab > 0 the step starts with the BF16 token-embedding gather
    (src/tts_native.c:490-493, 518-520) into its own output rows.
    """

    def __init__(self, cfg: LayerConfig, rows: int, row0: int = 0, seed: int = 1234,
                 device: str = "cuda", dtype: str = "bf16"):
        import torch
        self.cfg, self.rows, self.row0, self.device = cfg, rows, row0, device
        self.elem = 2 if dtype == "bf16" else 4
        T, D, I = rows, cfg.dim, cfg.inter
        bf = torch.bfloat16 if dtype == "bf16" else torch.float32
        e = lambda *s, dt=bf: torch.empty(s, dtype=dt, device=device)  # noqa: E731
        self.x, self.d_attn, self.d_ffn, self.y = e(T, D), e(T, D), e(T, D), e(T, D)
        self.q, self.k = e(T, cfg.n_q * cfg.head_dim), e(T, cfg.n_kv * cfg.head_dim)
        self.gate_up, self.act = e(T, 2 * I), e(T, I)
        f32 = torch.float32
        self.w_in, self.w_post = e(D, dt=f32), e(D, dt=f32)
        self.wq, self.wk = e(cfg.head_dim, dt=f32), e(cfg.head_dim, dt=f32)
        self.pos = e(T, dt=torch.int32)
        # global element offsets make each shard's data independent of the shard count
        for i, (t, width) in enumerate([(self.x, D), (self.d_attn, D), (self.d_ffn, D),
                                        (self.q, cfg.n_q * cfg.head_dim),
                                        (self.k, cfg.n_kv * cfg.head_dim), (self.gate_up, 2 * I)]):
            lai.synth_normal(t, seed=seed + i, offset=row0 * width)
        for i, w in enumerate([self.w_in, self.w_post, self.wq, self.wk]):
            lai.synth_normal(w, seed=seed + 100 + i, mean=1.0, std=0.02)
        if cfg.pos_mode == "random":
            lai.synth_uniform_i32(self.pos, seed=seed + 200, lo=0, hi=cfg.pos_period, offset=row0)
        else:
            self.pos.copy_((torch.arange(row0, row0 + T, device=device) % cfg.pos_period).to(torch.int32))
        table_pos = torch.arange(cfg.pos_period, dtype=torch.int32, device=device)
        self.cos, self.sin = lai.rope_table(table_pos, cfg.pos_period, cfg.head_dim, cfg.theta,
                                            device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        if cfg.vocab:
            self.table = e(cfg.vocab, D, dt=torch.bfloat16)
            lai.synth_normal(self.table, seed=seed + 300)
            self.ids = e(T, dt=torch.int32)
            lai.synth_uniform_i32(self.ids, seed=seed + 301, lo=0, hi=cfg.vocab, offset=row0)
            self.emb = e(T, D)
        self.kernel_names = cfg.kernels()

    def launches(self, stream=None):
        """The step as a list of callables, one kernel launch each."""
        c = self.cfg
        gfn = "lai_embed_gather_bf16" if self.elem == 2 else "lai_embed_gather_bf16_to_f32"
        gather = [lambda: lai.call(gfn, lai._p(self.emb), lai._p(self.table),
                                   lai._p(self.ids), self.rows, c.dim, c.vocab,
                                   lai._p(self.err), lai._s(stream))] if c.vocab else []
        return gather + [
            lambda: lai.add_rmsnorm(self.x, self.d_ffn, self.w_in, c.eps, y=self.y, stream=stream),
            lambda: lai.qk_norm_rope(self.q, self.k, self.wq, self.wk, self.cos, self.sin, self.pos,
                                     c.n_q, c.n_kv, c.head_dim, c.eps, err=self.err, stream=stream),
            lambda: lai.add_rmsnorm(self.x, self.d_attn, self.w_post, c.eps, y=self.y, stream=stream),
            lambda: lai.swiglu(self.gate_up, c.inter, out=self.act, stream=stream),
        ]

    def step(self, stream=None) -> None:
        for f in self.launches(stream):
            f()

    def bytes_per_launch(self) -> list[int]:
        b = self.cfg.bytes_per_token(self.elem)
        if self.elem == 4 and self.cfg.vocab:  # BF16 table row in, FP32 row out
            b = dict(b, embed_gather=2 * self.cfg.dim + 4 * self.cfg.dim + 4)
        return [b[k] * self.rows for k in self.kernel_names]


class SnakeSweep:
    """Vocoder SnakeBeta over the BigVGAN stages (config 4): x [batch, C, T] FP32 per
    stage, per-channel exp(alpha) / 1/exp(beta) pre-exponentiated as the reference
    does at load (src/tts_vocoder.c:221-227). One step = one launch per stage."""

    def __init__(self, stages=SNAKE_STAGES, batch=SNAKE_BATCH, seed: int = 77, device="cuda"):
        import torch
        self.stages, self.batch = list(stages), batch
        self.x, self.ea, self.ieb = [], [], []
        for i, (c, t) in enumerate(self.stages):
            x = torch.empty((batch, c, t), dtype=torch.float32, device=device)
            lai.synth_normal(x, seed=seed + i)
            a = torch.empty(c, dtype=torch.float32, device=device)
            b = torch.empty(c, dtype=torch.float32, device=device)
            lai.synth_normal(a, seed=seed + 100 + i, std=0.1)
            lai.synth_normal(b, seed=seed + 200 + i, std=0.1)
            self.x.append(x)
            self.ea.append(torch.exp(a))
            self.ieb.append(1.0 / torch.exp(b))
        self.kernel_names = tuple(f"snake_beta_{c}x{t}" for c, t in self.stages)

    def launches(self, stream=None):
        return [(lambda i=i: lai.snake_beta(self.x[i], self.ea[i], self.ieb[i], stream=stream))
                for i in range(len(self.stages))]

    def bytes_per_launch(self) -> list[int]:
        return [8 * self.batch * c * t for c, t in self.stages]  # FP32 read + write

    def rows_per_launch(self) -> list[int]:
        return [self.batch * c for c, _ in self.stages]


class VocResUnits:
    """The BigVGAN decoder's 12 ResUnits (config v1): per stage, x [batch, T, C] FP32
    channels-last and three units (dilations 1, 3, 9) with their own random weights:
    conv1 N(0,1)/sqrt(fan_in), conv2 0.1 N(0,1)/sqrt(fan_in), biases N(0,0.01), snake
    parameters pre-exponentiated from N(0,0.1). The small residual branch keeps the
    residual stream bounded, as a trained vocoder's is, although every timed step runs
    the units in place on the same x again: with conv2 at full scale x grows by about 2x
    per unit, passes 65536 within ~10 steps and moves SnakeBeta onto its full-range sinf
    path (40% slower) - a state no real input reaches. One step = one
    lai_voc_resunits_f32 call per stage (a snake1 kernel and two convolutions per unit)."""

    def __init__(self, stages=RESUNIT_STAGES, batch=RESUNIT_BATCH, passes: int = 3,
                 seed: int = 99, device="cuda"):
        import torch
        self.stages, self.batch, self.passes = list(stages), batch, passes
        self.x, self.units, self._keep = [], [], []
        k = 0

        def normal(shape, std=1.0):
            nonlocal k
            t = torch.empty(shape, dtype=torch.float32, device=device)
            lai.synth_normal(t, seed=seed + k, std=std)
            k += 1
            return t

        for c, t in self.stages:
            self.x.append(normal((batch, t, c)))
            params = []
            for d in RESUNIT_DILATIONS:
                params.append({
                    "ea1": torch.exp(normal(c, 0.1)), "ieb1": 1.0 / torch.exp(normal(c, 0.1)),
                    "w1": normal((c, c, 7), (7 * c) ** -0.5), "b1": normal(c, 0.01),
                    "ea2": torch.exp(normal(c, 0.1)), "ieb2": 1.0 / torch.exp(normal(c, 0.1)),
                    "w2": normal((c, c, 1), 0.1 * c ** -0.5), "b2": normal(c, 0.01),
                    "dilation": d})
            arr, keep = lai.voc_units(params)
            self.units.append(arr)
            self._keep.append((params, keep))
        n_max = max(batch * t * c for c, t in self.stages)
        self.scratch = torch.empty(4 * n_max, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.kernel_names = tuple(f"resunits_{c}x{t}" for c, t in self.stages)

    def launches(self, stream=None):
        return [(lambda i=i: lai.voc_resunits(self.x[i], self.units[i], self.scratch,
                                              self.passes, self.err, stream))
                for i in range(len(self.stages))]

    def flops_per_launch(self) -> list[float]:
        """FP32 convolution flops as the reference computes them: per unit and output
        element 2 * 7C (conv1) + 2 * C (conv2) multiply-adds."""
        return [16.0 * c * c * t * self.batch * len(RESUNIT_DILATIONS) for c, t in self.stages]

    def bytes_per_launch(self) -> list[int]:
        per = resunit_hbm_bytes_per_element(len(RESUNIT_DILATIONS), self.passes)
        return [per * self.batch * t * c for c, t in self.stages]

    def rows_per_launch(self) -> list[int]:
        return [self.batch * t for _, t in self.stages]  # time rows through 3 units


BIGVGAN_CHANNELS = (1536, 768, 384, 192, 96)  # src/tts_vocoder.c:245
BIGVGAN_RATES = (8, 5, 4, 3)                   # src/tts_vocoder.c:244


class VocDecoder:
    """The BigVGAN decoder after its init conv (config v2): 4 blocks, each SnakeBeta ->
    transposed conv (kernel 2r, stride r) -> 3 ResUnits, at the reference's own length
    progression T -> (T - 1) r (src/tts_vocoder.c:709-728): for t0 = 2000 (500 codec frames,
    40 s of audio) 1536 x 2000 -> 768 x 15992 -> 384 x 79955 -> 192 x 319816 -> 96 x 959445.
    Every step recomputes the decoder from the same input (no state carries over). Weights:
    transposed convs N(0,1)/sqrt(2 c_in), ResUnits as VocResUnits."""

    def __init__(self, t0: int = 2000, batch: int = 1, passes: int = 3, seed: int = 77,
                 device="cuda", x0=None):
        import torch
        self.t0, self.batch, self.passes = t0, batch, passes
        k = 0

        def normal(shape, std=1.0):
            nonlocal k
            t = torch.empty(shape, dtype=torch.float32, device=device)
            lai.synth_normal(t, seed=seed + k, std=std)
            k += 1
            return t

        self.x0 = normal((batch, t0, BIGVGAN_CHANNELS[0])) if x0 is None else x0
        self.blocks, self.outs, self.shapes = [], [], []
        t = t0
        scratch = 0
        for b, r in enumerate(BIGVGAN_RATES):
            c_in, c_out = BIGVGAN_CHANNELS[b], BIGVGAN_CHANNELS[b + 1]
            t_out = (t - 1) * r
            units = []
            for d in RESUNIT_DILATIONS:
                units.append({
                    "ea1": torch.exp(normal(c_out, 0.1)), "ieb1": 1.0 / torch.exp(normal(c_out, 0.1)),
                    "w1": normal((c_out, c_out, 7), (7 * c_out) ** -0.5), "b1": normal(c_out, 0.01),
                    "ea2": torch.exp(normal(c_out, 0.1)), "ieb2": 1.0 / torch.exp(normal(c_out, 0.1)),
                    "w2": normal((c_out, c_out, 1), 0.1 * c_out ** -0.5), "b2": normal(c_out, 0.01),
                    "dilation": d})
            self.blocks.append(lai.voc_block_params({
                "ea": torch.exp(normal(c_in, 0.1)), "ieb": 1.0 / torch.exp(normal(c_in, 0.1)),
                "w": normal((c_in, c_out, 2 * r), (2 * c_in) ** -0.5), "b": normal(c_out, 0.01),
                "rate": r, "units": units}))
            self.outs.append(torch.empty((batch, t_out, c_out), dtype=torch.float32, device=device))
            self.shapes.append((c_in, c_out, t, t_out, r))
            scratch = max(scratch, 2 * batch * t * c_in + 4 * batch * t_out * c_out)
            t = t_out
        self.scratch = torch.empty(scratch, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.kernel_names = tuple(f"block{b}_{c_in}to{c_out}x{t_out}"
                                  for b, (c_in, c_out, _, t_out, _) in enumerate(self.shapes))
        self.rows_step = batch * self.shapes[-1][3]  # audio samples (24 kHz) per step

    def launches(self, stream=None):
        def block(i):
            src = self.x0 if i == 0 else self.outs[i - 1]
            c_in, c_out, t, t_out, r = self.shapes[i]
            st = self.blocks[i][0]
            lai.call("lai_voc_bigvgan_block_f32", lai._p(self.outs[i]), lai._p(src),
                     lai._p(self.scratch), lai.ctypes.byref(st), self.batch, c_in, c_out, t,
                     self.passes, lai._p(self.err), lai._s(stream))
        return [(lambda i=i: block(i)) for i in range(len(self.shapes))]

    def flops_per_launch(self) -> list[float]:
        """F32 convolution flops: the transposed conv 2 * c_in * c_out * 2 per output row (two
        taps reach each output), the ResUnits 16 * c_out^2 per output row and unit."""
        return [self.batch * t_out * (4.0 * c_in * c_out + 16.0 * c_out * c_out * 3)
                for c_in, c_out, _, t_out, _ in self.shapes]

    def bytes_per_launch(self) -> list[int]:
        """Snake split of the input (read 4, write 8 per element); the transposed conv reads
        the 8-byte operand and writes x and the first unit's split input (12 per output
        element); the 3 ResUnits then move 112 per element (124 less the first split)."""
        return [self.batch * (20 * t * c_in + 124 * t_out * c_out)
                for c_in, c_out, t, t_out, _ in self.shapes]

    def rows_per_launch(self) -> list[int]:
        return [self.batch * t_out for _, _, _, t_out, _ in self.shapes]


class VocFullDecoder:
    """tts_vocoder_run from the pre-transformer's output to audio (config v3,
    src/tts_vocoder.c:658-758): 2 ConvNeXt upsample stages (transposed conv 1024 -> 1024,
    kernel = stride = 2, then the ConvNeXt block), the BigVGAN init conv 1024 -> 1536 (k=7),
    the 4 BigVGAN blocks (VocDecoder) and the final SnakeBeta -> conv 96 -> 1 -> clamp, for
    t_frames = 500 codec frames (40 s of audio): 1024 x 500 in, 959445 samples out, batch 1.
    Every step recomputes from the same input."""

    def __init__(self, t_frames: int = 500, batch: int = 1, passes: int = 3, seed: int = 88,
                 device="cuda", x_in=None):
        import torch
        self.batch, self.passes, self.t_frames = batch, passes, t_frames
        k = 0

        def normal(shape, std=1.0, mean=0.0):
            nonlocal k
            t = torch.empty(shape, dtype=torch.float32, device=device)
            lai.synth_normal(t, seed=seed + k, mean=mean, std=std)
            k += 1
            return t

        C = 1024
        self.x_in = normal((batch, t_frames, C)) if x_in is None else x_in
        self.ups = []
        t = t_frames
        for _ in range(2):
            self.ups.append({"w": lai.voc_pack_tconv(normal((C, C, 2), C ** -0.5), 2),
                             "b": normal(C, 0.01),
                             "cn": lai.voc_convnext_params({
                                 "dw_w": normal((C, 1, 7), 7 ** -0.5), "dw_b": normal(C, 0.01),
                                 "norm_w": normal(C, 0.1, 1.0), "norm_b": normal(C, 0.1),
                                 "pw1_w": normal((4 * C, C, 1), C ** -0.5),
                                 "pw1_b": normal(4 * C, 0.01),
                                 "pw2_w": normal((C, 4 * C, 1), (4 * C) ** -0.5),
                                 "pw2_b": normal(C, 0.01), "gamma": normal(C, 0.1)}),
                             "out": torch.empty((batch, 2 * t, C), dtype=torch.float32,
                                                device=device), "t": t})
            t *= 2
        self.t_dec = t
        self.init_w = lai.voc_pack_conv(normal((1536, C, 7), (7 * C) ** -0.5))
        self.init_b = normal(1536, 0.01)
        self.init_out = torch.empty((batch, t, 1536), dtype=torch.float32, device=device)
        self.dec = VocDecoder(t0=t, batch=batch, passes=passes, seed=seed + 1000, device=device,
                              x0=self.init_out)
        self.fin = {"ea": torch.exp(normal(96, 0.1)), "ieb": 1.0 / torch.exp(normal(96, 0.1)),
                    "w": normal((1, 96, 7), (96 * 7) ** -0.5), "b": normal(1, 0.01)}
        self.t_final = self.dec.shapes[-1][3]
        self.audio = torch.empty((batch, self.t_final), dtype=torch.float32, device=device)
        self.scratch = self.dec.scratch  # the largest need (the last block's) covers every stage
        self.err = self.dec.err
        self.kernel_names = ("upsample0_tconv", "upsample0_convnext", "upsample1_tconv",
                             "upsample1_convnext", "init_conv") + self.dec.kernel_names + ("final",)
        self.rows_step = batch * self.t_final

    def launches(self, stream=None):
        L = []
        src = self.x_in
        for u in self.ups:
            def tconv(u=u, src=src):
                lai.call("lai_voc_conv_transpose1d_f32", lai._p(u["out"]), lai._p(src),
                         lai._p(self.scratch), lai._p(u["w"]), lai._p(u["b"]), self.batch, 1024,
                         1024, u["t"], 2, 2, self.passes, lai._p(self.err), lai._s(stream))
            L.append(tconv)
            L.append(lambda u=u: lai.voc_convnext(u["out"], u["cn"], self.scratch, self.passes,
                                                  self.err, stream))
            src = u["out"]

        def init(src=src):
            lai.call("lai_voc_conv1d_f32", lai._p(self.init_out), lai._p(src), lai._p(self.scratch),
                     lai._p(self.init_w), lai._p(self.init_b), self.batch, 1024, 1536, self.t_dec,
                     7, 1, self.passes, lai._p(self.err), lai._s(stream))
        L.append(init)
        L += self.dec.launches(stream)
        L.append(lambda: lai.voc_final(self.dec.outs[-1], self.fin["ea"], self.fin["ieb"],
                                       self.fin["w"], self.fin["b"], out=self.audio, stream=stream))
        return L

    def flops_per_launch(self) -> list[float]:
        C, B = 1024, self.batch
        f = []
        for u in self.ups:
            f += [2.0 * C * C * 2 * u["t"] * B, 16.0 * C * C * 2 * u["t"] * B]
        f.append(2.0 * C * 1536 * 7 * self.t_dec * B)
        f += self.dec.flops_per_launch()
        f.append(2.0 * 96 * 7 * self.t_final * B)
        return f

    def bytes_per_launch(self) -> list[int]:
        C, B = 1024, self.batch
        b = []
        for u in self.ups:
            b += [B * (12 * u["t"] * C + 4 * 2 * u["t"] * C), 92 * B * 2 * u["t"] * C]
        b.append(B * self.t_dec * (12 * C + 4 * 1536))
        b += self.dec.bytes_per_launch()
        b.append(B * self.t_final * (4 * 96 + 4))
        return b

    def rows_per_launch(self) -> list[int]:
        B = self.batch
        r = []
        for u in self.ups:
            r += [B * 2 * u["t"], B * 2 * u["t"]]
        r.append(B * self.t_dec)
        r += self.dec.rows_per_launch()
        r.append(B * self.t_final)
        return r


RVQ_CODEBOOKS, RVQ_SIZE, RVQ_DIM, RVQ_OUT = 16, 2048, 256, 512
PRE_CONV_OUT, PRE_CONV_KERNEL = 1024, 3
XFMR_LAYERS, XFMR_HIDDEN, XFMR_ATTN, XFMR_HEADS, XFMR_HD, XFMR_INTER = 8, 512, 1024, 16, 64, 1024
XFMR_EPS, XFMR_THETA = 1e-5, 10000.0


class VocFront:
    """tts_vocoder_run stages 1-3 (src/tts_vocoder.c:589-640) on the device, channels-last:
    codes [T, 16] int64 -> RVQ decode (rvq_decode, :428-455: 16 codebook lookups [2048, 256]
    each projected 256 -> 512 and summed) -> pre_conv CausalConv1d 512 -> 1024, k = 3
    (:612-616) -> the 8-layer pre-transformer (voc_pre_transformer,
    src/tts_vocoder_xfmr.c:126-225: input_proj 1024 -> 512 + bias; per layer RMSNorm, q/k/v
    512 -> 1024, NeoX RoPE (theta 1e4), causal attention over 16 heads of 64, o 1024 -> 512
    with LayerScale + residual, RMSNorm, SwiGLU MLP 512 -> 1024 -> 512 with LayerScale +
    residual; final RMSNorm, output_proj 512 -> 1024 + bias) -> y [T, 1024], the layout
    VocFullDecoder takes. The reference transposes [C, T] <-> [T, C] around the transformer;
    channels-last throughout needs no transpose.

    Device form: RVQ is one gather of the 16 codebook rows of a frame side by side ([T, 4096])
    and one GEMM against the 16 projections laid side by side (K = 4096), which sums the
    codebooks inside the accumulator; q|k|v and gate|up are each one GEMM over the
    concatenated (gate/up row-interleaved) weights; attention reads q, k, v out of the q|k|v
    output with RoPE folded in; o and down add their LayerScale'd output into the residual in
    the GEMM epilogue. All linears are 3xTF32 tcgen05 GEMMs (F32 parity). Weights in the
    reference's layouts are kept in `ref` for the checker."""

    def __init__(self, t_frames: int = 500, passes: int = 3, seed: int = 99, device="cuda"):
        import torch
        self.t, self.passes = t_frames, passes
        T = t_frames
        k = 0

        def normal(shape, std=1.0, mean=0.0):
            nonlocal k
            t = torch.empty(shape, dtype=torch.float32, device=device)
            lai.synth_normal(t, seed=seed + k, mean=mean, std=std)
            k += 1
            return t

        f32 = dict(dtype=torch.float32, device=device)
        codes = torch.empty((T, RVQ_CODEBOOKS), dtype=torch.int32, device=device)
        lai.synth_uniform_i32(codes, seed + 500, 0, RVQ_SIZE)
        self.codes = codes.to(torch.int64)
        H, A, I = XFMR_HIDDEN, XFMR_ATTN, XFMR_INTER
        ref = {"codebooks": normal((RVQ_CODEBOOKS, RVQ_SIZE, RVQ_DIM)),
               "proj": normal((RVQ_CODEBOOKS, RVQ_OUT, RVQ_DIM), RVQ_DIM ** -0.5 / 4),
               "pre_w": normal((PRE_CONV_OUT, RVQ_OUT, PRE_CONV_KERNEL), (3 * RVQ_OUT) ** -0.5),
               "pre_b": normal(PRE_CONV_OUT, 0.01),
               "in_w": normal((H, PRE_CONV_OUT), PRE_CONV_OUT ** -0.5), "in_b": normal(H, 0.01),
               "final_norm": normal(H, 0.1, 1.0),
               "out_w": normal((PRE_CONV_OUT, H), H ** -0.5), "out_b": normal(PRE_CONV_OUT, 0.01),
               "layers": []}
        for _ in range(XFMR_LAYERS):
            ref["layers"].append({
                "in_norm": normal(H, 0.1, 1.0), "wq": normal((A, H), H ** -0.5),
                "wk": normal((A, H), H ** -0.5), "wv": normal((A, H), H ** -0.5),
                "wo": normal((H, A), A ** -0.5), "attn_ls": normal(H, 0.1),
                "post_norm": normal(H, 0.1, 1.0), "gate": normal((I, H), H ** -0.5),
                "up": normal((I, H), H ** -0.5), "down": normal((H, I), I ** -0.5),
                "mlp_ls": normal(H, 0.1)})
        self.ref = ref
        pk = lambda w: lai.voc_pack_conv(w if w.dim() == 3 else w.unsqueeze(-1))  # noqa: E731
        # the 16 projections side by side: W[o, cb*256 + d] = proj[cb][o, d]
        self.rvq_w = pk(ref["proj"].permute(1, 0, 2).reshape(RVQ_OUT, RVQ_CODEBOOKS * RVQ_DIM))
        self.pre_w, self.in_w, self.out_w = pk(ref["pre_w"]), pk(ref["in_w"]), pk(ref["out_w"])
        self.layers = []
        for L in ref["layers"]:
            gu = torch.stack([L["gate"], L["up"]], dim=1).reshape(2 * I, H)  # rows g0,u0,g1,u1..
            self.layers.append({"qkv": pk(torch.cat([L["wq"], L["wk"], L["wv"]])), "gu": pk(gu),
                                "o": pk(L["wo"]), "down": pk(L["down"])})
        self.zeros = torch.zeros(3 * A, **f32)
        pos = torch.arange(T, dtype=torch.int32, device=device)
        self.cos, self.sin = lai.rope_table(pos, T, XFMR_HD, XFMR_THETA, device=device)
        self.g = torch.empty((T, RVQ_CODEBOOKS * RVQ_DIM), **f32)
        self.rvq = torch.empty((1, T, RVQ_OUT), **f32)
        self.pre = torch.empty((1, T, PRE_CONV_OUT), **f32)
        self.x = torch.empty((T, H), **f32)
        self.xn = torch.empty((T, H), **f32)
        self.qkv = torch.empty((T, 3 * A), **f32)
        self.attn = torch.empty((T, A), **f32)
        self.gu = torch.empty((T, 2 * I), **f32)
        self.ffn = torch.empty((T, I), **f32)
        self.y = torch.empty((1, T, PRE_CONV_OUT), **f32)
        self.scratch = torch.empty(2 * T * RVQ_CODEBOOKS * RVQ_DIM, **f32)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.kernel_names = ("rvq_gather", "rvq_proj", "pre_conv", "input_proj") + tuple(
            f"layer{i}_{n}" for i in range(XFMR_LAYERS)
            for n in ("norm1", "qkv", "attention", "o_scale_residual", "norm2", "gate_up",
                      "swiglu", "down_scale_residual")) + ("final_norm", "output_proj")
        self.rows_step = T

    def _conv(self, out, x, w, bias, c_in, c_out, kernel, stream):
        lai.call("lai_voc_conv1d_f32", lai._p(out), lai._p(x), lai._p(self.scratch), lai._p(w),
                 lai._p(bias), 1, c_in, c_out, self.t, kernel, 1, self.passes, lai._p(self.err),
                 lai._s(stream))

    def _scale_res(self, inp, w, gamma, c_in, stream):
        lai.call("lai_voc_linear_scale_residual_f32", lai._p(self.x), lai._p(inp),
                 lai._p(self.scratch), lai._p(w), lai._p(self.zeros), lai._p(gamma), self.t, c_in,
                 XFMR_HIDDEN, self.passes, lai._p(self.err), lai._s(stream))

    def launches(self, stream=None):
        T, H, A, I = self.t, XFMR_HIDDEN, XFMR_ATTN, XFMR_INTER
        r = self.ref
        L = [lambda: lai.call("lai_voc_rvq_gather_f32", lai._p(self.g), lai._p(r["codebooks"]),
                              lai._p(self.codes), T, RVQ_CODEBOOKS, RVQ_SIZE, RVQ_DIM,
                              lai._p(self.err), lai._s(stream)),
             lambda: self._conv(self.rvq, self.g, self.rvq_w, self.zeros,
                                RVQ_CODEBOOKS * RVQ_DIM, RVQ_OUT, 1, stream),
             lambda: self._conv(self.pre, self.rvq, self.pre_w, r["pre_b"], RVQ_OUT,
                                PRE_CONV_OUT, PRE_CONV_KERNEL, stream),
             lambda: self._conv(self.x, self.pre, self.in_w, r["in_b"], PRE_CONV_OUT, H, 1,
                                stream)]
        for R, W in zip(r["layers"], self.layers):
            L += [lambda R=R: lai.rmsnorm(self.x, R["in_norm"], XFMR_EPS, y=self.xn, stream=stream),
                  lambda W=W: self._conv(self.qkv, self.xn, W["qkv"], self.zeros, H, 3 * A, 1,
                                         stream),
                  lambda: lai.prefill_attention_rope(self.qkv, XFMR_HEADS, XFMR_HEADS, XFMR_HD,
                                                     self.cos, self.sin, out=self.attn,
                                                     stream=stream),
                  lambda R=R, W=W: self._scale_res(self.attn, W["o"], R["attn_ls"], A, stream),
                  lambda R=R: lai.rmsnorm(self.x, R["post_norm"], XFMR_EPS, y=self.xn,
                                          stream=stream),
                  lambda W=W: self._conv(self.gu, self.xn, W["gu"], self.zeros, H, 2 * I, 1,
                                         stream),
                  lambda: lai.swiglu(self.gu, I, out=self.ffn, stream=stream),
                  lambda R=R, W=W: self._scale_res(self.ffn, W["down"], R["mlp_ls"], I, stream)]
        L += [lambda: lai.rmsnorm(self.x, r["final_norm"], XFMR_EPS, y=self.xn, stream=stream),
              lambda: self._conv(self.y, self.xn, self.out_w, r["out_b"], H, PRE_CONV_OUT, 1,
                                 stream)]
        return L

    def flops_per_launch(self) -> list[float]:
        T, H, A, I = self.t, XFMR_HIDDEN, XFMR_ATTN, XFMR_INTER
        f = [0.0, 2.0 * T * RVQ_CODEBOOKS * RVQ_DIM * RVQ_OUT,
             2.0 * T * RVQ_OUT * PRE_CONV_OUT * PRE_CONV_KERNEL, 2.0 * T * PRE_CONV_OUT * H]
        attn = 2.0 * 2 * XFMR_HEADS * XFMR_HD * T * (T + 1) / 2  # q.k and p.v over keys <= t
        f += [0.0, 2.0 * T * H * 3 * A, attn, 2.0 * T * A * H, 0.0, 2.0 * T * H * 2 * I, 0.0,
              2.0 * T * I * H] * XFMR_LAYERS
        return f + [0.0, 2.0 * T * H * PRE_CONV_OUT]

    def bytes_per_launch(self) -> list[int]:
        T, H, A, I = self.t, XFMR_HIDDEN, XFMR_ATTN, XFMR_INTER
        G = RVQ_CODEBOOKS * RVQ_DIM
        conv = lambda ci, co, k: 4 * (T * ci + T * co + 2 * k * co * ci + co)  # noqa: E731
        b = [T * RVQ_CODEBOOKS * 8 + 2 * 4 * T * G, conv(G, RVQ_OUT, 1),
             conv(RVQ_OUT, PRE_CONV_OUT, PRE_CONV_KERNEL), conv(PRE_CONV_OUT, H, 1)]
        b += [4 * (2 * T * H + H), conv(H, 3 * A, 1), 4 * (T * 3 * A + 2 * T * XFMR_HD + T * A),
              conv(A, H, 1) + 4 * (T * H + H), 4 * (2 * T * H + H), conv(H, 2 * I, 1),
              4 * (T * 2 * I + T * I), conv(I, H, 1) + 4 * (T * H + H)] * XFMR_LAYERS
        return b + [4 * (2 * T * H + H), conv(H, PRE_CONV_OUT, 1)]

    def rows_per_launch(self) -> list[int]:
        return [self.t] * len(self.kernel_names)


class VocCodesToAudio:
    """The whole tts_vocoder_run on the device (config v4, src/tts_vocoder.c:589-758):
    VocFront (codes -> pre-transformer output) then VocFullDecoder (-> audio) on the front's
    output buffer; for 500 codec frames (40 s of audio) 500 x 16 codes in, 959445 samples
    out. Every step recomputes from the same codes."""

    def __init__(self, t_frames: int = 500, passes: int = 3, seed: int = 99, device="cuda"):
        self.front = VocFront(t_frames, passes=passes, seed=seed, device=device)
        self.dec = VocFullDecoder(t_frames, batch=1, passes=passes, seed=seed + 5000,
                                  device=device, x_in=self.front.y)
        self.codes, self.audio, self.t_frames = self.front.codes, self.dec.audio, t_frames
        self.kernel_names = self.front.kernel_names + self.dec.kernel_names
        self.rows_step = self.dec.rows_step
        self.err = self.front.err
        self.graph = None

    def launches(self, stream=None):
        return self.front.launches(stream) + self.dec.launches(stream)

    def run(self, graph: bool = False):
        """codes -> audio once. graph: replay the ~150 launches as one CUDA graph (captured on
        first use; the codes and audio buffers stay where they are, so new codes copied into
        `codes` are picked up by the next replay)."""
        import torch
        if not graph:
            for f in self.launches():
                f()
            return self.audio
        if self.graph is None:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                for f in self.launches():
                    f()
        self.graph.replay()
        return self.audio

    def flops_per_launch(self) -> list[float]:
        return self.front.flops_per_launch() + self.dec.flops_per_launch()

    def bytes_per_launch(self) -> list[int]:
        return self.front.bytes_per_launch() + self.dec.bytes_per_launch()

    def rows_per_launch(self) -> list[int]:
        return self.front.rows_per_launch() + self.dec.rows_per_launch()


class VocConvNeXt:
    """The vocoder's two ConvNeXt upsample blocks (config n1): C = 1024 at 2 T0 and 4 T0
    time rows (T0 = 500 codec frames, src/tts_vocoder.c:658-670), batch 8, FP32
    channels-last; weights random at trained-model scale (depthwise N(0,1)/sqrt 7,
    pointwise N(0,1)/sqrt(fan_in), LayerNorm 1+N(0,0.1) / N(0,0.1), biases N(0,0.01),
    layer scale N(0,0.1): the block adds a small update, so repeated in-place steps keep
    x bounded). One step = one lai_voc_convnext_f32 call per stage (3 launches each)."""

    def __init__(self, stages=((1024, 1000), (1024, 2000)), batch=8, passes: int = 3,
                 seed: int = 555, device="cuda"):
        import torch
        self.stages, self.batch, self.passes = list(stages), batch, passes
        k = 0

        def normal(shape, std=1.0, mean=0.0):
            nonlocal k
            t = torch.empty(shape, dtype=torch.float32, device=device)
            lai.synth_normal(t, seed=seed + k, mean=mean, std=std)
            k += 1
            return t

        self.x, self.params = [], []
        for c, t in self.stages:
            self.x.append(normal((batch, t, c)))
            self.params.append(lai.voc_convnext_params({
                "dw_w": normal((c, 1, 7), 7 ** -0.5), "dw_b": normal(c, 0.01),
                "norm_w": normal(c, 0.1, 1.0), "norm_b": normal(c, 0.1),
                "pw1_w": normal((4 * c, c, 1), c ** -0.5), "pw1_b": normal(4 * c, 0.01),
                "pw2_w": normal((c, 4 * c, 1), (4 * c) ** -0.5), "pw2_b": normal(c, 0.01),
                "gamma": normal(c, 0.1)}))
        n_max = max(batch * t * c for c, t in self.stages)
        self.scratch = torch.empty(10 * n_max, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.kernel_names = tuple(f"convnext_{c}x{t}" for c, t in self.stages)

    def launches(self, stream=None):
        return [(lambda i=i: lai.voc_convnext(self.x[i], self.params[i], self.scratch,
                                              self.passes, self.err, stream))
                for i in range(len(self.stages))]

    def flops_per_launch(self) -> list[float]:
        """The two pointwise convolutions: 2 * (C * 4C + 4C * C) flops per time row."""
        return [16.0 * c * c * t * self.batch for c, t in self.stages]

    def bytes_per_launch(self) -> list[int]:
        """Per element of x: depthwise+LayerNorm reads 4 and writes the 8-byte operand;
        pw1 reads 8 and writes 32 (h is 4C wide, hi/lo); pw2 reads 32 and x, writes x."""
        per = 92 if self.passes == 3 else 48
        return [per * self.batch * t * c for c, t in self.stages]

    def rows_per_launch(self) -> list[int]:
        return [self.batch * t for _, t in self.stages]


class SampleBatch:
    """Token sampling of config s3: `rows` decode rows of codec logits (vocab 3072,
    src/tts_native.c:1096-1099) with repetition penalty over 64-token histories, top-k 50,
    temperature 0.9. One step = one lai_sample_topk_f32 launch."""

    def __init__(self, rows: int = 256, vocab: int = 3072, top_k: int = 50, temperature=0.9,
                 penalty=1.05, hist: int = 64, seed: int = 31, device="cuda"):
        import torch
        self.rows, self.vocab, self.top_k = rows, vocab, top_k
        self.temperature, self.penalty = temperature, penalty
        self.logits = torch.empty((rows, vocab), dtype=torch.float32, device=device)
        lai.synth_normal(self.logits, seed=seed, std=2.0)
        self.history = torch.empty((rows, hist), dtype=torch.int32, device=device)
        lai.synth_uniform_i32(self.history, seed + 1, 0, vocab)
        self.hist_len = torch.full((rows,), hist, dtype=torch.int32, device=device)
        self.u = torch.empty(rows, dtype=torch.float32, device=device)
        lai.synth_normal(self.u, seed=seed + 2, std=0.25, mean=0.5)
        self.u.clamp_(0.0, 1.0)
        self.out = torch.empty(rows, dtype=torch.int32, device=device)
        self.kernel_names = ("sample_topk",)

    def launches(self, stream=None):
        return [lambda: lai.sample_topk(self.logits, self.u, self.temperature, self.top_k,
                                        self.history, self.hist_len, self.penalty,
                                        out=self.out, stream=stream)]

    def bytes_per_launch(self) -> list[int]:
        return [self.rows * (self.vocab * 4 + self.history.shape[1] * 4 + 8)]

    def rows_per_launch(self) -> list[int]:
        return [self.rows]


class DecodeAttention:
    """Decode attention of config a3: `seqs` sequences x 1 token at seeded random
    positions 0..max_seq-1, GQA n_heads / n_kv_heads, head_dim 128, F32 KV cache
    [seqs, max_seq, n_kv*128] filled with N(0,1). One step = lai_decode_attention_f32:
    append each token's k/v at its position and attend over keys 0..pos."""

    def __init__(self, seqs: int = 256, n_heads: int = 16, n_kv_heads: int = 8,
                 max_seq: int = 4096, seed: int = 4242, device="cuda"):
        import torch
        self.seqs, self.n_heads, self.n_kv, self.max_seq = seqs, n_heads, n_kv_heads, max_seq
        kv_dim = n_kv_heads * 128

        def normal(shape, k):
            t = torch.empty(shape, dtype=torch.float32, device=device)
            lai.synth_normal(t, seed=seed + k)
            return t

        self.q = normal((seqs, n_heads * 128), 0)
        self.k_new, self.v_new = normal((seqs, kv_dim), 1), normal((seqs, kv_dim), 2)
        self.k_cache = normal((seqs, max_seq, kv_dim), 3)
        self.v_cache = normal((seqs, max_seq, kv_dim), 4)
        self.pos = torch.empty(seqs, dtype=torch.int32, device=device)
        lai.synth_uniform_i32(self.pos, seed + 5, 0, max_seq)
        self.out = torch.empty_like(self.q)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.scratch = lai.decode_attention_scratch(seqs, n_heads, n_kv_heads, max_seq, device)
        self.keys = int((self.pos.to(torch.int64) + 1).sum().item())
        self.kernel_names = ("decode_attention",)

    def launches(self, stream=None):
        return [lambda: lai.decode_attention(self.q, self.k_new, self.v_new, self.k_cache,
                                             self.v_cache, self.pos, self.n_heads, self.n_kv,
                                             self.scratch, out=self.out, err=self.err,
                                             stream=stream)]

    def bytes_per_launch(self) -> list[int]:
        """K and V rows 0..pos read once per (sequence, kv head); q, the new k/v and the
        output once; the appended cache rows written."""
        kv_dim = self.n_kv * 128
        return [self.keys * kv_dim * 4 * 2 + self.seqs * (2 * self.n_heads * 128 + 4 * kv_dim) * 4]

    def rows_per_launch(self) -> list[int]:
        return [self.seqs]


class DecodeLinear:
    """The decode step's linear path through `layers` decoder layers
    (src/tts_native.c:637-668 per layer), fused per layer: RMSNorm+QKV GEMV, O GEMV +
    residual, RMSNorm + gate/up GEMV + SwiGLU, down GEMV + residual. FP32 activations,
    BF16 weights (q, k, v rows concatenated into one matrix, gate/up rows interleaved
    as the reference's fused weight), every layer its own weights so a step streams
    them all from HBM. The attention output is a fixed stand-in (attention is not part
    of this path)."""

    # weight bytes per element and the entry points' format names (the reference's GPU modes)
    WEIGHT_BYTES = {"bf16": 2, "f16": 2, "i8": 1, "f32": 4}

    def __init__(self, cfg: DecodeConfig, seed: int = 4321, device: str = "cuda",
                 wfmt: str = "bf16", chain: bool = False):
        import torch
        self.cfg, self.rows, self.wfmt = cfg, cfg.m, wfmt
        self.chain, self.form = None, "per-op"
        self.wbytes = self.WEIGHT_BYTES[wfmt]
        D, I, M = cfg.dim, cfg.inter, cfg.m
        self.qkv_n = cfg.q_dim + 2 * cfg.kv_dim
        f32, bf = torch.float32, torch.bfloat16
        self.scales = {}  # id(weight) -> per-row scales (INT8)

        def w(n, k, s):
            t = torch.empty((n, k), dtype=bf, device=device)
            t = lai.synth_normal(t, seed=seed + s, std=float(k) ** -0.5)
            if wfmt == "f16":
                return lai.convert_bf16_to_f16(t)
            if wfmt == "f32":
                return t.float()
            if wfmt == "i8":
                q, sc = lai.quantize_rows_i8(t)
                self.scales[id(q)] = sc
                return q
            return t

        L = cfg.layers
        self.Wqkv = [w(self.qkv_n, D, 10 * l + 1) for l in range(L)]
        self.Wo = [w(D, cfg.q_dim, 10 * l + 2) for l in range(L)]
        self.Wgu = [w(2 * I, D, 10 * l + 3) for l in range(L)]
        self.Wd = [w(D, I, 10 * l + 4) for l in range(L)]
        self.w_in = lai.synth_normal(torch.empty(D, dtype=f32, device=device), seed=seed + 5,
                                     mean=1.0, std=0.02)
        self.w_post = lai.synth_normal(torch.empty(D, dtype=f32, device=device), seed=seed + 6,
                                       mean=1.0, std=0.02)
        self.x = lai.synth_normal(torch.empty((M, D), dtype=f32, device=device), seed=seed + 7)
        self.attn = lai.synth_normal(torch.empty((M, cfg.q_dim), dtype=f32, device=device),
                                     seed=seed + 8)
        self.qkv = torch.empty((M, self.qkv_n), dtype=f32, device=device)
        self.act = torch.empty((M, I), dtype=f32, device=device)
        if chain:  # the step also as one persistent kernel (lai_gemv_chain_*)
            if wfmt != "bf16" or M != 1:
                raise ValueError("the GEMV chain takes BF16 weights at M = 1")
            self.chain = lai.GemvChain(self.chain_ops())
            self.form = "chain"

    PER_OP_NAMES = ("rmsnorm_qkv_gemv", "o_gemv_residual", "rmsnorm_gate_up_gemv_swiglu",
                    "down_gemv_residual")

    @property
    def kernel_names(self):
        return ("gemv_chain",) if self.form == "chain" else self.PER_OP_NAMES * self.cfg.layers

    def set_form(self, form: str):
        """"chain" (one persistent kernel per step) or "per-op" (one launch per projection)."""
        if form == "chain" and self.chain is None:
            raise ValueError("built without the chain")
        self.form = form

    def chain_ops(self):
        """The step's 4 * layers GEMVs as chain ops, in the order per_op_launches() runs them."""
        c = self.cfg
        x, a, qkv, act = self.x[0], self.attn[0], self.qkv[0], self.act[0]
        ops = []
        for l in range(c.layers):
            ops += [(lai.CHAIN_STORE, self.Wqkv[l], x, self.w_in, qkv, c.eps),
                    (lai.CHAIN_RESIDUAL, self.Wo[l], a, None, x, 0.0),
                    (lai.CHAIN_SWIGLU, self.Wgu[l], x, self.w_post, act, c.eps),
                    (lai.CHAIN_RESIDUAL, self.Wd[l], act, None, x, 0.0)]
        return ops

    def launches(self, stream=None):
        if self.form == "chain":
            return [lambda: self.chain.run(stream)]
        return self.per_op_launches(stream)

    def per_op_launches(self, stream=None):
        """One fused-GEMV launch per projection (4 per layer)."""
        c = self.cfg
        sc = lambda W: self.scales.get(id(W))  # noqa: E731
        out = []
        for l in range(c.layers):
            out += [
                lambda l=l: lai.gemv(self.x, self.Wqkv[l], self.w_in, c.eps, y=self.qkv,
                                     stream=stream, scales=sc(self.Wqkv[l])),
                lambda l=l: lai.gemv_residual(self.x, self.attn, self.Wo[l], stream=stream,
                                              scales=sc(self.Wo[l])),
                lambda l=l: lai.gemv_swiglu(self.x, self.Wgu[l], self.w_post, c.eps, out=self.act,
                                            stream=stream, scales=sc(self.Wgu[l])),
                lambda l=l: lai.gemv_residual(self.x, self.act, self.Wd[l], stream=stream,
                                              scales=sc(self.Wd[l])),
            ]
        return out

    def unfused_library_launches(self):
        """The same step as separate kernels around cuBLAS GEMMs in the weights' own type
        (torch), every intermediate through HBM: the library baseline the fusion is measured
        against. None for INT8 weights, which cuBLAS does not take as they are stored."""
        import torch.nn.functional as F
        c = self.cfg
        if self.wfmt == "i8":
            return None
        wt = self.Wqkv[0].dtype

        def layer(l):
            def qkv():
                xn = lai.rmsnorm(self.x, self.w_in, c.eps)
                self.qkv.copy_(F.linear(xn.to(wt), self.Wqkv[l]))

            def o():
                lai.add(self.x, F.linear(self.attn.to(wt), self.Wo[l]).float())

            def gu():
                xn = lai.rmsnorm(self.x, self.w_post, c.eps)
                lai.swiglu(F.linear(xn.to(wt), self.Wgu[l]).float(), c.inter, out=self.act)

            def down():
                lai.add(self.x, F.linear(self.act.to(wt), self.Wd[l]).float())
            return [qkv, o, gu, down]
        return [f for l in range(c.layers) for f in layer(l)]

    def bytes_per_launch(self) -> list[int]:
        """Weights (wbytes per element, plus 4 bytes of scale per row for INT8) + activations."""
        c, M, e = self.cfg, self.cfg.m, self.wbytes
        D, I = c.dim, c.inter
        s = 4 if self.wfmt == "i8" else 0
        per = [self.qkv_n * (D * e + s) + M * D * 4 + M * self.qkv_n * 4 + D * 4,
               D * (c.q_dim * e + s) + M * c.q_dim * 4 + 2 * M * D * 4,
               2 * I * (D * e + s) + M * D * 4 + M * I * 4 + D * 4,
               D * (I * e + s) + M * I * 4 + 2 * M * D * 4] * c.layers
        return [sum(per)] if self.form == "chain" else per

    def rows_per_launch(self) -> list[int]:
        return [self.cfg.m] * len(self.kernel_names)


@dataclasses.dataclass(frozen=True)
class TtsConfig:
    """Shapes of run_decode_loop's per-frame work (src/tts_native.h:29-56). Defaults: the
    Qwen3-TTS 0.6B talker (hidden 1024, FFN 3072, 28 layers) and its 5-layer code predictor
    of the same width (mtp_project is then a copy, src/tts_native.c:88-99)."""
    name: str = "qwen3-tts-0.6b"
    hidden: int = 1024
    inter: int = 3072
    layers: int = 28
    cp_inter: int = 3072
    cp_layers: int = 5
    n_q: int = 16
    n_kv: int = 8
    head_dim: int = 128
    talker_vocab: int = 3072
    codec_vocab: int = 2048
    groups: int = 16
    suppress_start: int = 2048
    eos: int = 2150
    max_seq: int = 4096
    eps: float = 1e-6
    theta: float = 1e6
    temperature: float = 0.9
    top_k: int = 50
    penalty: float = 1.05


class TtsFrame:
    """One frame of run_decode_loop (src/tts_native.c:1042-1165) on the device, every step a
    library call on one stream and every sampled token kept in device memory:

      talker_forward(codec_sum) (:608-686): per layer RMSNorm + fused q|k|v GEMV, per-head
        q/k RMSNorm + RoPE at the cache position + cache append + attention (one launch),
        o GEMV + residual,
        RMSNorm + gate/up GEMV + SwiGLU, down GEMV + residual; final RMSNorm (the hidden state
        the code predictor starts from) and the codec head GEMV -> 3072 logits;
      logits [2048, 3072) except EOS -> -1e9, repetition penalty over the cb0 history, top-k
        sampling -> cb0, appended to the history (:1092-1105);
      the code predictor (:1110-1149): its input rows are the talker hidden state, cb0's codec
        embedding, then each sub-code's embedding; for j = 0..14 the 5-layer transformer's last
        row -> RMSNorm -> lm_head[j] -> top-k -> sub-code j + 1 -> embedding (talker space)
        added into codec_sum;
      codec_sum += the trailing text embedding (:1152-1156), the next frame's input.

    The reference re-runs the code predictor over all rows for every sub-code
    (code_predictor_forward, :689-760, no cache). Attention is causal, so the last row's
    output depends only on the rows before it: this runs each row once against a 16-row KV
    cache and gets the same result for the row that feeds lm_head[j] (15 + 1 row-steps per
    frame instead of 2 + 3 + ... + 16 = 135).

    Weights are synthetic BF16 (q, k, v rows concatenated; gate/up rows interleaved as the
    reference's fused weight), norms ~1 + N(0, 0.02). The uniform draws are taken in order
    from `draws` (16 per frame: cb0, then sub-codes 1..15), as rand() would be.
    """

    def __init__(self, cfg: TtsConfig, frames: int, seed: int = 77, device: str = "cuda"):
        import torch
        self.cfg, self.frames, self.device = cfg, frames, device
        c = cfg
        H, qd, kvd = c.hidden, c.n_q * c.head_dim, c.n_kv * c.head_dim
        self.qd, self.kvd = qd, kvd
        bf, f32 = torch.bfloat16, torch.float32
        g = torch.Generator(device=device).manual_seed(seed)

        def w(n, k, scale=None):
            t = torch.randn((n, k), generator=g, device=device) * (scale or k ** -0.5)
            return t.to(bf)

        def nrm(n):
            return (1.0 + 0.02 * torch.randn(n, generator=g, device=device)).to(f32)

        def layer(inter):
            return {"wqkv": w(qd + 2 * kvd, H), "wo": w(H, qd), "wgu": w(2 * inter, H),
                    "wd": w(H, inter), "in_norm": nrm(H), "post_norm": nrm(H),
                    "q_norm": nrm(c.head_dim), "k_norm": nrm(c.head_dim)}

        self.talker = [layer(c.inter) for _ in range(c.layers)]
        self.final_norm = nrm(H)
        self.codec_head = w(c.talker_vocab, H)
        self.codec_embed = w(c.talker_vocab, H, 0.5)
        self.cp = [layer(c.cp_inter) for _ in range(c.cp_layers)]
        self.cp_norm = nrm(H)
        self.cp_heads = [w(c.codec_vocab, H) for _ in range(c.groups - 1)]
        self.cp_embed = [w(c.codec_vocab, H, 0.5) for _ in range(c.groups - 1)]
        self.trailing = (0.5 * torch.randn((frames, H), generator=g, device=device)).to(f32)
        self.draws = torch.rand((frames, c.groups), generator=g, device=device)
        # caches, tables, buffers
        self.kc = [torch.zeros((1, c.max_seq, kvd), dtype=f32, device=device)
                   for _ in range(c.layers)]
        self.vc = [torch.zeros_like(k) for k in self.kc]
        self.cp_kc = [torch.zeros((1, c.groups, kvd), dtype=f32, device=device)
                      for _ in range(c.cp_layers)]
        self.cp_vc = [torch.zeros_like(k) for k in self.cp_kc]
        pos_all = torch.arange(c.max_seq, dtype=torch.int32, device=device)
        self.cos, self.sin = lai.rope_table(pos_all, c.max_seq, c.head_dim, c.theta,
                                            device=device)
        self.cp_pos = torch.arange(c.groups, dtype=torch.int32, device=device)
        self.scr = lai.decode_attention_scratch(1, c.n_q, c.n_kv, c.max_seq, device)
        self.cp_scr = lai.decode_attention_scratch(1, c.n_q, c.n_kv, c.groups, device)
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        self.x = torch.zeros((1, H), dtype=f32, device=device)
        self.qkv = torch.empty((1, qd + 2 * kvd), dtype=f32, device=device)
        self.attn = torch.empty((1, qd), dtype=f32, device=device)
        self.act = torch.empty((1, max(c.inter, c.cp_inter)), dtype=f32, device=device)
        self.logits = torch.empty((1, c.talker_vocab), dtype=f32, device=device)
        self.cp_logits = torch.empty((1, c.codec_vocab), dtype=f32, device=device)
        self.codec_sum = (0.5 * torch.randn((1, H), generator=g, device=device)).to(f32)
        self.codes = torch.zeros((frames, c.groups), dtype=torch.int32, device=device)
        self.history = torch.zeros((1, frames), dtype=torch.int32, device=device)
        self.hist_len = torch.zeros(1, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        # the frame body reads and writes only these fixed buffers, so it can be captured
        # once as a CUDA graph and replayed for every frame
        self.u_frame = torch.zeros((1, c.groups), dtype=f32, device=device)
        self.trail_frame = torch.zeros((1, H), dtype=f32, device=device)
        self.codes_frame = torch.zeros((1, c.groups), dtype=torch.int32, device=device)
        self.frame_idx = 0
        self.record = None  # list: logits before each sampling (tests)
        self.graph = None

    def _layers(self, layers, kc, vc, pos, scr, inter, stream):
        c = self.cfg
        q = self.qkv[:, :self.qd]
        k = self.qkv[:, self.qd:self.qd + self.kvd]
        v = self.qkv[:, self.qd + self.kvd:]
        act = self.act[:, :inter]
        for i, L in enumerate(layers):
            lai.gemv(self.x, L["wqkv"], L["in_norm"], c.eps, y=self.qkv, stream=stream)
            # per-head q/k RMSNorm + RoPE at pos, cache append and attention: one launch
            lai.decode_attention(q, k, v, kc[i], vc[i], pos, c.n_q, c.n_kv, scratch=scr,
                                 out=self.attn, err=self.err, stream=stream,
                                 qk=(L["q_norm"], L["k_norm"], self.cos, self.sin, c.eps))
            lai.gemv_residual(self.x, self.attn, L["wo"], stream=stream)
            lai.gemv_swiglu(self.x, L["wgu"], L["post_norm"], c.eps, out=act, stream=stream)
            lai.gemv_residual(self.x, act, L["wd"], stream=stream)

    def _sample(self, logits, j, history, stream):
        c = self.cfg
        if self.record is not None:
            self.record.append(logits.clone())
        out = self.codes_frame[:, j]
        u = self.u_frame[:, j]
        if history:
            lai.sample_topk(logits, u, c.temperature, c.top_k, self.history, self.hist_len,
                            c.penalty, out=out, stream=stream)
        else:
            lai.sample_topk(logits, u, c.temperature, c.top_k, out=out, stream=stream)
        return out

    def _gather(self, table, ids, stream):  # one embedding row into x
        lai.call("lai_embed_gather_bf16_to_f32", lai._p(self.x), lai._p(table), lai._p(ids),
                 1, self.cfg.hidden, table.shape[0], lai._p(self.err), lai._s(stream))

    def frame(self, graph: bool = False, staged: bool = False):
        """Run one frame; its 16 codes land in codes[frame] (and codes_frame). graph: replay
        the frame body as one CUDA graph (captured on first use) instead of launching its ~750
        kernels. staged: the caller has already put this frame's 16 draws and trailing
        embedding into u_frame and trail_frame."""
        import torch
        f = self.frame_idx
        if f >= self.frames:
            raise RuntimeError("frame capacity reached")
        if not staged:
            self.u_frame.copy_(self.draws[f:f + 1])
            self.trail_frame.copy_(self.trailing[f:f + 1])
        if not graph:
            self._body(None)
        else:
            if self.graph is None:
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self._body(None)
                # capture records without running: replay for this frame
            self.graph.replay()
        self.codes[f:f + 1].copy_(self.codes_frame)
        self.frame_idx += 1

    def _body(self, stream):
        c = self.cfg
        # talker step on codec_sum at the cache position
        self.x.copy_(self.codec_sum)
        self._layers(self.talker, self.kc, self.vc, self.pos, self.scr, c.inter, stream)
        lai.rmsnorm(self.x, self.final_norm, c.eps, y=self.x, stream=stream)  # hidden state
        lai.gemv(self.x, self.codec_head, y=self.logits, stream=stream)
        lai.logits_mask_range(self.logits, c.suppress_start, c.talker_vocab, keep=c.eos,
                              stream=stream)
        cb0 = self._sample(self.logits, 0, True, stream)
        lai.history_append(self.history, self.hist_len, cb0, err=self.err, stream=stream)
        # code predictor: row 0 = the hidden state (already in x), row 1 = cb0's embedding,
        # then each sub-code's; an embedding is gathered straight into x, the row's input
        self._layers(self.cp, self.cp_kc, self.cp_vc, self.cp_pos[0:1], self.cp_scr,
                     c.cp_inter, stream)
        self._gather(self.codec_embed, cb0, stream)
        self.codec_sum.copy_(self.x)
        for j in range(c.groups - 1):
            self._layers(self.cp, self.cp_kc, self.cp_vc, self.cp_pos[j + 1:j + 2], self.cp_scr,
                         c.cp_inter, stream)
            # final RMSNorm of the row folded into lm_head[j]'s GEMV
            lai.gemv(self.x, self.cp_heads[j], self.cp_norm, c.eps, y=self.cp_logits,
                     stream=stream)
            sub = self._sample(self.cp_logits, j + 1, False, stream)
            self._gather(self.cp_embed[j], sub, stream)
            lai.add(self.codec_sum, self.x, stream=stream)
        lai.add(self.codec_sum, self.trail_frame, stream=stream)
        self.pos.add_(1)

    def launches_per_frame(self) -> int:
        """Library kernels per frame (the 2 tensor copies and the position add not counted)."""
        c = self.cfg
        per_layer = 5
        return (c.layers * per_layer + 2 + 3 + c.groups * c.cp_layers * per_layer + 1
                + (c.groups - 1) * 4 + 1)

    def weight_bytes_per_frame(self) -> int:
        """Weights streamed from HBM per frame: every talker layer once, every code-predictor
        layer once per row (16 rows), the codec head once, the 15 lm_heads once each."""
        c = self.cfg
        H, qd, kvd = c.hidden, self.qd, self.kvd

        def layer(inter):
            return 2 * ((qd + 2 * kvd) * H + H * qd + 2 * inter * H + H * inter)
        return (c.layers * layer(c.inter) + c.groups * c.cp_layers * layer(c.cp_inter)
                + 2 * c.talker_vocab * H + (c.groups - 1) * 2 * c.codec_vocab * H)


class TtsDecode:
    """Config d1: run_decode_loop frames of the Qwen3-TTS 0.6B talker + code predictor
    (TtsFrame with TtsConfig defaults), one frame per step, each replayed as one CUDA graph.
    Rows are frames (16 codec codes each, 80 ms of 24 kHz audio at 12.5 frames/s)."""

    def __init__(self, frames: int, seed: int = 77, device: str = "cuda"):
        self.cfg = TtsConfig()
        self.tf = TtsFrame(self.cfg, frames, seed=seed, device=device)
        self.kernel_names = ("tts_frame",)
        self.err = self.tf.err

    def launches(self, stream=None):
        return [lambda: self.tf.frame(graph=True)]

    def bytes_per_launch(self) -> list[int]:
        return [self.tf.weight_bytes_per_frame()]

    def rows_per_launch(self) -> list[int]:
        return [1]
