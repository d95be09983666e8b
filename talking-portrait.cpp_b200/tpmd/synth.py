"""Seeded synthetic inputs for the motion decoder (motion_dec).

The reference's decoder benchmarks run on a real portrait and real weights,
which are not redistributable; these generators stand in for them with the
same shapes and value distributions (random-init LIA/StyleGAN decoder):

* raw weights: conv and modulation weights N(0, 1); modulation biases 1.0
  (EqualLinear bias_init=1, the StyleGAN2 convention); every other bias 0 by
  default (`bias_std` > 0 draws them N(0, bias_std) instead, which parity
  tests use so the bias paths are exercised); blur / upsample kernels
  [1,3,3,1] x [1,3,3,1], normalised, x4 (the up-sampling gain);
  dec.input.input N(0, 1) [1, 512, 4, 4].
* feats: the source-portrait feature pyramid, N(0, 1) maps [ST_OC[j], r*r]
  (channel-last, pixel-major) for r = 8 << j.
* styles: latent = w_src + Q @ alpha with w_src ~ N(0, 1)^512, Q the
  orthonormal factor of a seeded N(0, 1) [512, 20] matrix, alpha ~ N(0, 0.5)
  (0.5 is the standard deviation). For frame sequences alpha follows a random
  walk with N(0, 0.05) steps clipped to [-3, 3].

Tensor names and torch shapes are those of the reference's motion_ae GGUF
(src/motion_dec.cpp:17-29, 267-272, 357-433, 829-883). `fold` applies the
load-time scale folding (motion_ae_scale, src/motion_enc.cpp:14-45) exactly as
the reference loader does: f32 data times (float) scale
(src/gguf_load.cpp:178-183).
"""
from __future__ import annotations

import numpy as np

ST_IC = (512, 512, 512, 512, 256, 128, 64)
ST_OC = (512, 512, 512, 256, 128, 64, 32)
STYLE_DIM = 512
N_DIRS = 20


def blur_kernel4() -> np.ndarray:
    k1 = np.array([1, 3, 3, 1], np.float32)
    k = np.outer(k1, k1)
    return (k / k.sum() * 4.0).astype(np.float32)


def tensor_shapes() -> dict[str, tuple[int, ...]]:
    """name -> torch shape (leading singleton of 5-D modconv weights squeezed)."""
    s: dict[str, tuple[int, ...]] = {"dec.input.input": (1, 512, 4, 4)}

    def modconv(base, ic, oc, k, blur):
        s[base + ".conv.weight"] = (oc, ic, k, k)
        s[base + ".conv.modulation.weight"] = (ic, STYLE_DIM)
        s[base + ".conv.modulation.bias"] = (ic,)
        if blur:
            s[base + ".conv.blur.kernel"] = (4, 4)

    modconv("dec.conv1", 512, 512, 3, False)
    s["dec.conv1.activate.bias"] = (1, 512, 1, 1)
    for i in range(14):
        j, up = i // 2, i % 2 == 0
        ic, oc = (ST_IC[j] if up else ST_OC[j]), ST_OC[j]
        modconv(f"dec.convs.{i}", ic, oc, 3, up)
        s[f"dec.convs.{i}.activate.bias"] = (1, oc, 1, 1)
    for j in range(7):
        oc = ST_OC[j]
        modconv(f"dec.to_flows.{j}", oc, 3, 1, False)
        s[f"dec.to_flows.{j}.bias"] = (1, 3, 1, 1)
        s[f"dec.to_flows.{j}.upsample.kernel"] = (4, 4)
        s[f"dec.to_rgbs.{j}.conv.0.weight"] = (3, oc, 1, 1)
        s[f"dec.to_rgbs.{j}.conv.1.bias"] = (1, 3, 1, 1)
        s[f"dec.to_rgbs.{j}.bias"] = (1, 3, 1, 1)
        s[f"dec.to_rgbs.{j}.upsample.kernel"] = (4, 4)
    return s


def ggml_ne(shape: tuple[int, ...]) -> tuple[int, int, int, int]:
    """ggml dims (fastest first) of a torch shape, padded to 4."""
    ne = tuple(reversed(shape))
    return tuple(list(ne) + [1] * (4 - len(ne)))[:4]


def make_weights(seed: int = 0, bias_std: float = 0.0, flow_gain: float = 1.0) -> dict[str, np.ndarray]:
    """Raw (unfolded) f32 weights in torch shapes.

    flow_gain scales the ToFlow conv weights. 1.0 is the plain random init,
    whose flow maps are large (|fl| ~ 2-5), saturate tanh and move every
    sampling point by up to half the image; the decoder is then so sensitive
    that the reference's own f16 arithmetic ends at SSIM ~0.95 against its
    fp32 output. 0.25 keeps the flows in tanh's linear range, as a trained
    model's are; parity gates use it (PARITY_FLOW_GAIN)."""
    rng = np.random.default_rng([seed, 1])
    out: dict[str, np.ndarray] = {}
    bk = blur_kernel4()
    for name, shape in tensor_shapes().items():
        if name.endswith(".kernel"):
            out[name] = bk.copy()
        elif name.endswith("modulation.bias"):
            out[name] = np.ones(shape, np.float32)
        elif name.endswith("bias"):
            out[name] = (rng.standard_normal(shape, np.float32) * np.float32(bias_std)
                         if bias_std > 0 else np.zeros(shape, np.float32))
        else:
            out[name] = rng.standard_normal(shape, np.float32)
            if name.startswith("dec.to_flows.") and name.endswith(".conv.weight"):
                out[name] *= np.float32(flow_gain)
    return out


PARITY_FLOW_GAIN = 0.25


def fold(raw: dict[str, np.ndarray], scale_for) -> dict[str, np.ndarray]:
    """Apply motion_ae_scale: each tensor times (float) scale_for(name, ne)."""
    return {n: (a.astype(np.float32) * np.float32(scale_for(n, ggml_ne(a.shape))))
            for n, a in raw.items()}


def make_feats(seed: int = 0, smooth: bool = True) -> list[np.ndarray]:
    """feats[j]: [r*r, ST_OC[j]] float32 (channel-last), r = 8 << j.

    smooth=True (default): per channel, N(0, 1) white noise low-pass filtered
    by a periodic Gaussian of standard deviation r/16 pixels and renormalised
    to zero mean and unit variance, i.e. N(0, 1) maps with the spatial
    correlation an encoder's feature pyramid has. smooth=False: white noise.
    White-noise maps make the decoder chaotic: the bilinear warp of an
    uncorrelated map turns a grid rounding error of e (normalised units) into
    an error of about e*r/2 in the sampled value, so rounding grows roughly
    tenfold per level and two float32 formulations of the same graph end at a
    frame cosine near 0.9. Parity gates are therefore evaluated on smooth
    maps; throughput does not depend on the values.
    """
    rng = np.random.default_rng([seed, 2])
    out = []
    for j in range(7):
        r, c = 8 << j, ST_OC[j]
        x = rng.standard_normal((c, r, r))
        if smooth:
            f = np.fft.fftfreq(r)
            sig = r / 16.0
            g = np.exp(-2.0 * (np.pi * sig) ** 2 * (f[:, None] ** 2 + f[None, :] ** 2))
            x = np.fft.ifft2(np.fft.fft2(x) * g).real
            x = (x - x.mean(axis=(1, 2), keepdims=True)) / x.std(axis=(1, 2), keepdims=True)
        out.append(np.ascontiguousarray(x.reshape(c, r * r).T).astype(np.float32))
    return out


def make_basis(seed: int = 0) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng([seed, 3])
    w_src = rng.standard_normal(STYLE_DIM).astype(np.float32)
    q, _ = np.linalg.qr(rng.standard_normal((STYLE_DIM, N_DIRS)))
    return w_src, q.astype(np.float32)


def styles_config0(seed: int = 0, n: int = 1) -> np.ndarray:
    """n independent frames: latent = w_src + Q @ alpha, alpha ~ N(0, 0.5)."""
    w_src, q = make_basis(seed)
    rng = np.random.default_rng([seed, 4])
    alpha = rng.standard_normal((n, N_DIRS)).astype(np.float32) * np.float32(0.5)
    return (w_src[None, :] + alpha @ q.T).astype(np.float32)


def styles_walk(seed: int = 0, n: int = 50, clip: int = 0) -> np.ndarray:
    """A clip of n frames whose alpha is a seeded random walk: start
    N(0, 0.5), steps N(0, 0.05), clipped to [-3, 3]."""
    w_src, q = make_basis(seed)
    rng = np.random.default_rng([seed, 5, clip])
    a = rng.standard_normal(N_DIRS).astype(np.float32) * np.float32(0.5)
    steps = rng.standard_normal((n, N_DIRS)).astype(np.float32) * np.float32(0.05)
    alphas = np.empty((n, N_DIRS), np.float32)
    for t in range(n):
        if t:
            a = np.clip(a + steps[t], -3.0, 3.0).astype(np.float32)
        alphas[t] = a
    return (w_src[None, :] + alphas @ q.T).astype(np.float32)


ENC_IN = (32, 64, 128, 256, 512, 512, 512)
ENC_OUT = (64, 128, 256, 512, 512, 512, 512)


def encoder_shapes() -> dict[str, tuple[int, ...]]:
    """name -> torch shape of the motion encoder's tensors (enc.* and the
    baked direction basis dec.direction.Q), src/motion_enc.cpp:46-140."""
    p = "enc.net_app.convs."
    s: dict[str, tuple[int, ...]] = {p + "0.0.weight": (32, 3, 1, 1), p + "0.1.bias": (1, 32, 1, 1)}
    for i in range(1, 8):
        c, co = ENC_IN[i - 1], ENC_OUT[i - 1]
        b = f"{p}{i}."
        s[b + "conv1.0.weight"] = (c, c, 3, 3)
        s[b + "conv1.1.bias"] = (1, c, 1, 1)
        s[b + "conv2.0.kernel"] = (4, 4)
        s[b + "conv2.1.weight"] = (co, c, 3, 3)
        s[b + "conv2.2.bias"] = (1, co, 1, 1)
        s[b + "skip.0.kernel"] = (4, 4)
        s[b + "skip.1.weight"] = (co, c, 1, 1)
    s[p + "8.weight"] = (512, 512, 4, 4)
    for i in range(5):
        out = 20 if i == 4 else 512
        s[f"enc.fc.{i}.weight"] = (out, 512)
        s[f"enc.fc.{i}.bias"] = (out,)
    s["dec.direction.Q"] = (512, 20)
    return s


def make_encoder_weights(seed: int = 0, bias_std: float = 0.1) -> dict[str, np.ndarray]:
    """Raw (unfolded) encoder weights: N(0,1) conv and linear weights (the
    Equal* convention: the runtime scale is 1/sqrt(fan_in)), N(0, bias_std)
    biases, the normalised [1,3,3,1] outer-product blur (sum 1, as the
    downsampling Blur uses it), Q with orthonormal columns (QR of a seeded
    N(0,1) [512, 20] matrix)."""
    rng = np.random.default_rng([seed, 7])
    k1 = np.array([1, 3, 3, 1], np.float64)
    k = np.outer(k1, k1)
    k = (k / k.sum()).astype(np.float32)
    out: dict[str, np.ndarray] = {}
    for name, shape in encoder_shapes().items():
        if name.endswith(".kernel"):
            out[name] = k.copy()
        elif name == "dec.direction.Q":
            q, _ = np.linalg.qr(rng.standard_normal(shape))
            out[name] = q.astype(np.float32)
        elif name.endswith(".bias"):
            out[name] = (rng.standard_normal(shape) * bias_std).astype(np.float32)
        else:
            out[name] = rng.standard_normal(shape).astype(np.float32)
    return out


def make_image(seed: int = 0) -> np.ndarray:
    """A smooth synthetic portrait-sized image [3, 512, 512] in [-1, 1]: a
    few random low-frequency cosines per channel plus mild noise."""
    rng = np.random.default_rng([seed, 8])
    yy, xx = np.meshgrid(np.arange(512) / 512.0, np.arange(512) / 512.0, indexing="ij")
    img = np.zeros((3, 512, 512), np.float64)
    for c in range(3):
        for _ in range(6):
            fx, fy = rng.uniform(0.5, 6.0, 2)
            ph = rng.uniform(0, 2 * np.pi)
            img[c] += rng.uniform(0.1, 0.3) * np.cos(2 * np.pi * (fx * xx + fy * yy) + ph)
        img[c] += 0.05 * rng.standard_normal((512, 512))
    return np.clip(img, -1.0, 1.0).astype(np.float32)


# The flow-matching transformer of config 4 (8 blocks, d = 1024, 16 heads,
# banded attention, 9 Euler steps, 3-way CFG, 50-frame chunks with 10-frame
# context); keys as the GGUF's float.fmt.* hyper-parameters.
FMT_CONFIG = dict(dim_h=1024, depth=8, n_heads=16, dim_w=512, dim_a=512, dim_e=7, chunk_frames=50,
                  prev_frames=10, attn_window=2, t_freq_dim=256, nfe=10, mlp_ratio=4.0, ln_eps=1e-6,
                  a_cfg=2.0, e_cfg=1.0)
# a small instance of the same architecture for fast parity tests
FMT_SMALL = dict(FMT_CONFIG, dim_h=256, depth=2, n_heads=4)


def fmt_shapes(cfg: dict) -> dict[str, tuple[int, ...]]:
    """name -> torch shape of the FMT tensors (src/fmt.cpp:64-170)."""
    H, T = cfg["dim_h"], cfg["chunk_frames"] + cfg["prev_frames"]
    CD, FF = cfg["dim_w"] + cfg["dim_a"] + cfg["dim_e"], int(cfg["dim_h"] * cfg["mlp_ratio"])
    s: dict[str, tuple[int, ...]] = {}

    def lin(n, out, inp):
        s[n + ".weight"] = (out, inp)
        s[n + ".bias"] = (out,)
    lin("t_embedder.mlp.0", H, cfg["t_freq_dim"])
    lin("t_embedder.mlp.2", H, H)
    lin("c_embedder", H, CD)
    lin("x_embedder.proj", H, cfg["dim_w"])
    s["pos_embed"] = (1, T, H)
    for i in range(cfg["depth"]):
        b = f"blocks.{i}."
        lin(b + "adaLN_modulation.1", 6 * H, H)
        lin(b + "attn.qkv", 3 * H, H)
        lin(b + "attn.proj", H, H)
        lin(b + "mlp.fc1", FF, H)
        lin(b + "mlp.fc2", H, FF)
    lin("decoder.adaLN_modulation.1", 2 * H, H)
    lin("decoder.linear", cfg["dim_w"], H)
    return s


def make_fmt_weights(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    """Random-init FMT weights: Linear weights N(0, 1/fan_in) (activations
    stay O(1); the adaLN layers are not zero-initialised, so every block
    contributes), biases N(0, 0.02), pos_embed N(0, 0.1)."""
    rng = np.random.default_rng([seed, 11])
    out: dict[str, np.ndarray] = {}
    for n, sh in fmt_shapes(cfg).items():
        if n == "pos_embed":
            out[n] = (rng.standard_normal(sh) * 0.1).astype(np.float32)
        elif n.endswith(".bias"):
            out[n] = (rng.standard_normal(sh) * 0.02).astype(np.float32)
        else:
            out[n] = (rng.standard_normal(sh) / np.sqrt(sh[1])).astype(np.float32)
    return out


def make_fmt_chunk(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    """Inputs of one sampler chunk (chunk_io, src/pipeline.cpp:15-33):
    reference latent wr, previous-context audio features and motion, the
    chunk's audio features, the initial noise x0; emotion 'happy' (index 3)."""
    rng = np.random.default_rng([seed, 12])
    D, P, CF = cfg["dim_w"], cfg["prev_frames"], cfg["chunk_frames"]
    f = lambda *sh: rng.standard_normal(sh).astype(np.float32)
    return dict(wr=f(D), prev_wa=f(P, D), cond_audio=f(CF, D), prev_x=f(P, D), x0=f(CF, D), emotion=3)


# wav2vec2-base as config 4 names it (7-conv group-norm stem, 12 layers,
# d = 768, 12 heads, FFN 3072) with the projection to the 512-d motion space;
# keys as the GGUF's float.audio.* hyper-parameters (src/audio_enc.cpp:25-45)
AUDIO_CONFIG = dict(n_layers=12, n_heads=12, hidden=768, ffn=3072, dim_w=512, ln_eps=1e-5,
                    conv_dim=(512,) * 7, conv_kernel=(10, 3, 3, 3, 3, 2, 2), conv_stride=(5, 2, 2, 2, 2, 2, 2),
                    pos_kernel=128, pos_groups=16, sample_rate=16000, fps=25)
AUDIO_SMALL = dict(AUDIO_CONFIG, n_layers=2, n_heads=4, hidden=128, ffn=256, dim_w=64, conv_dim=(32,) * 7,
                   pos_kernel=16, pos_groups=4)


def audio_shapes(cfg: dict) -> dict[str, tuple[int, ...]]:
    """name -> torch shape of the audio encoder's tensors."""
    s: dict[str, tuple[int, ...]] = {}
    ic = 1
    for i in range(7):
        s[f"feature_extractor.conv_layers.{i}.conv.weight"] = (cfg["conv_dim"][i], ic, cfg["conv_kernel"][i])
        ic = cfg["conv_dim"][i]
    s["feature_extractor.conv_layers.0.layer_norm.weight"] = (cfg["conv_dim"][0],)
    s["feature_extractor.conv_layers.0.layer_norm.bias"] = (cfg["conv_dim"][0],)
    C, H, F, L = cfg["conv_dim"][6], cfg["hidden"], cfg["ffn"], cfg["n_layers"]
    s["feature_projection.layer_norm.weight"] = (C,)
    s["feature_projection.layer_norm.bias"] = (C,)
    s["feature_projection.projection.weight"] = (H, C)
    s["feature_projection.projection.bias"] = (H,)
    s["encoder.pos_conv_embed.conv.weight"] = (H, H // cfg["pos_groups"], cfg["pos_kernel"])
    s["encoder.pos_conv_embed.conv.bias"] = (H,)
    s["encoder.layer_norm.weight"] = (H,)
    s["encoder.layer_norm.bias"] = (H,)
    for i in range(L):
        b = f"encoder.layers.{i}."
        for pj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            s[b + f"attention.{pj}.weight"] = (H, H)
            s[b + f"attention.{pj}.bias"] = (H,)
        s[b + "layer_norm.weight"] = (H,)
        s[b + "layer_norm.bias"] = (H,)
        s[b + "feed_forward.intermediate_dense.weight"] = (F, H)
        s[b + "feed_forward.intermediate_dense.bias"] = (F,)
        s[b + "feed_forward.output_dense.weight"] = (H, F)
        s[b + "feed_forward.output_dense.bias"] = (H,)
        s[b + "final_layer_norm.weight"] = (H,)
        s[b + "final_layer_norm.bias"] = (H,)
    s["audio_projection.0.weight"] = (cfg["dim_w"], H * L)
    s["audio_projection.0.bias"] = (cfg["dim_w"],)
    s["audio_projection.1.weight"] = (cfg["dim_w"],)
    s["audio_projection.1.bias"] = (cfg["dim_w"],)
    return s


def make_audio_weights(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    """Random-init audio encoder: conv and linear weights N(0, 1/fan_in),
    biases N(0, 0.02), layer-norm gains 1 + N(0, 0.1) and shifts N(0, 0.1)."""
    rng = np.random.default_rng([seed, 13])
    out: dict[str, np.ndarray] = {}
    for n, sh in audio_shapes(cfg).items():
        if "norm" in n:
            base = 1.0 if n.endswith(".weight") else 0.0
            out[n] = (base + rng.standard_normal(sh) * 0.1).astype(np.float32)
        elif n.endswith(".bias"):
            out[n] = (rng.standard_normal(sh) * 0.02).astype(np.float32)
        else:
            fan = int(np.prod(sh[1:]))
            out[n] = (rng.standard_normal(sh) / np.sqrt(fan)).astype(np.float32)
    return out


def make_audio(seconds: float, seed: int = 0, sr: int = 16000) -> np.ndarray:
    """Config-4 style synthetic speech-like audio: band-limited noise
    (80-4000 Hz) under a 2-8 Hz syllabic envelope, peak 0.5, then the
    feature extractor's zero-mean unit-variance normalisation."""
    rng = np.random.default_rng([seed, 14])
    n = int(seconds * sr)
    spec = np.fft.rfft(rng.standard_normal(n))
    f = np.fft.rfftfreq(n, 1.0 / sr)
    spec[(f < 80) | (f > 4000)] = 0
    x = np.fft.irfft(spec, n)
    t = np.arange(n) / sr
    env = 0.5 + 0.5 * np.sin(2 * np.pi * rng.uniform(2, 8) * t + rng.uniform(0, 2 * np.pi))
    x = x * env
    x = 0.5 * x / np.abs(x).max()
    return ((x - x.mean()) / (x.std() + 1e-7)).astype(np.float32)
# the small audio encoder with the 512-d output the sampler's audio condition takes
AUDIO_SMALL512 = dict(AUDIO_SMALL, dim_w=512)

