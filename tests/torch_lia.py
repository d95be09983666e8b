"""An independent float64 formulation of the motion decoder in torch (CPU),
used only to cross-check the oracle's graph composition.

It is written from the module definitions the reference's graph implements
(StyleGAN2 / LIA Synthesis as described by src/motion_dec.cpp:794-888 and
the folding notes of src/motion_enc.cpp:14-45), deliberately in the
*unfolded* form: RAW weights with the Equal* runtime scales applied at run
time, weight-side modulation and demodulation (w' = w*s,
d = rsqrt(sum w'^2 + 1e-8)), FusedLeakyReLU as sqrt(2)*lrelu(x + b), the
up-conv as torch.conv_transpose2d(stride 2) followed by Blur(pad 1, 1), the
skip up-sampling as upfirdn2d(up=2, pad=(2,1)) and the warp as
torch.nn.functional.grid_sample. None of the oracle's derived tensors (S_aug,
tsubcf, folded scales) are used.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

ST_IC = (512, 512, 512, 512, 256, 128, 64)
ST_OC = (512, 512, 512, 256, 128, 64, 32)


def _t(a):
    return torch.as_tensor(np.asarray(a), dtype=torch.float64)


def _upfirdn(x, k, up, pad0, pad1):
    """x [1, C, H, W]; zero-stuff by `up`, pad (pad0, pad1), correlate with k"""
    c = x.shape[1]
    if up > 1:
        n, _, h, w = x.shape
        z = torch.zeros(n, c, h * up, w * up, dtype=x.dtype)
        z[:, :, ::up, ::up] = x
        x = z
    x = F.pad(x, (pad0, pad1, pad0, pad1))
    kk = k.flip([0, 1])[None, None].repeat(c, 1, 1, 1)  # upfirdn2d convolves
    return F.conv2d(x, kk, groups=c)


class TorchLIA:
    def __init__(self, raw: dict, feats: list):
        self.w = {k: _t(v) for k, v in raw.items()}
        # feats[j]: [r*r, C] channel-last -> [1, C, r, r]
        self.feats = [_t(f).T.reshape(1, f.shape[1], 8 << j, 8 << j) for j, f in enumerate(feats)]

    def _style(self, base, lat):
        W = self.w[base + ".modulation.weight"]
        b = self.w[base + ".modulation.bias"]
        return lat @ (W * (1.0 / math.sqrt(W.shape[1]))).T + b

    def _modconv(self, x, base, lat, demod=True, up=False):
        W = self.w[base + ".weight"]  # [OC, IC, k, k]
        oc, ic, k, _ = W.shape
        s = self._style(base, lat)
        w = W * (1.0 / math.sqrt(ic * k * k)) * s[None, :, None, None]
        if demod:
            d = torch.rsqrt((w ** 2).sum([1, 2, 3]) + 1e-8)
            w = w * d[:, None, None, None]
        if up:
            y = F.conv_transpose2d(x, w.transpose(0, 1), stride=2)
            return _upfirdn(y, self.w[base + ".blur.kernel"], 1, 1, 1)
        return F.conv2d(x, w, padding=k // 2)

    @staticmethod
    def _flrelu(x, b):
        return math.sqrt(2.0) * F.leaky_relu(x + b.reshape(1, -1, 1, 1), 0.2)

    def decode(self, latent: np.ndarray) -> np.ndarray:
        lat = _t(latent)
        x = self.w["dec.input.input"]
        x = self._flrelu(self._modconv(x, "dec.conv1.conv", lat), self.w["dec.conv1.activate.bias"])
        skip = skip_f = None
        for j in range(7):
            r = 8 << j
            b1, b2 = f"dec.convs.{2 * j}", f"dec.convs.{2 * j + 1}"
            x = self._flrelu(self._modconv(x, b1 + ".conv", lat, up=True),
                             self.w[b1 + ".activate.bias"])
            out = self._flrelu(self._modconv(x, b2 + ".conv", lat), self.w[b2 + ".activate.bias"])
            bf, br = f"dec.to_flows.{j}", f"dec.to_rgbs.{j}"
            fl = self._modconv(out, bf + ".conv", lat, demod=False) + self.w[bf + ".bias"]
            if skip_f is not None:
                fl = fl + _upfirdn(skip_f, self.w[bf + ".upsample.kernel"], 2, 2, 1)
            skip_f = fl
            lin = torch.linspace(-1.0, 1.0, r, dtype=torch.float64)
            gx = torch.tanh(fl[0, 0]) + lin[None, :]
            gy = torch.tanh(fl[0, 1]) + lin[:, None]
            m = torch.sigmoid(fl[0, 2])
            grid = torch.stack([gx, gy], -1)[None]
            sampled = F.grid_sample(self.feats[j], grid, mode="bilinear", padding_mode="zeros",
                                    align_corners=False)
            warp = sampled * m
            trunk = warp + out * (1 - m)
            Wr = self.w[br + ".conv.0.weight"]
            rgb = F.conv2d(warp, Wr * (1.0 / math.sqrt(Wr.shape[1])))
            rgb = self._flrelu(rgb, self.w[br + ".conv.1.bias"]) + self.w[br + ".bias"].reshape(1, 3, 1, 1)
            if skip is not None:
                rgb = rgb + _upfirdn(skip, self.w[br + ".upsample.kernel"], 2, 2, 1)
            skip = rgb
            x = trunk
        return skip[0].numpy()


ENC_IN = (32, 64, 128, 256, 512, 512, 512)
ENC_OUT = (64, 128, 256, 512, 512, 512, 512)


class TorchEncoder:
    """The LIA appearance encoder (EncoderApp) + fc chain + direction, in
    float64 torch and the unfolded form: RAW weights with the EqualConv2d /
    EqualLinear runtime scales 1/sqrt(fan_in) applied at run time,
    FusedLeakyReLU as sqrt(2)*lrelu(x + b), ResBlock output (main + skip) /
    sqrt(2), Blur as upfirdn2d with pads (2, 2) before the stride-2 3x3 conv
    and (1, 1) before the stride-2 1x1 skip conv (the graph of
    src/motion_enc.cpp:46-184 before its load-time folding)."""

    def __init__(self, raw: dict):
        self.w = {k: _t(v) for k, v in raw.items()}

    def _conv(self, x, name, stride=1, pad=0):
        W = self.w[name]
        fan = W.shape[1] * W.shape[2] * W.shape[3]
        return F.conv2d(x, W * (1.0 / math.sqrt(fan)), stride=stride, padding=pad)

    @staticmethod
    def _flrelu(x, b):
        return math.sqrt(2.0) * F.leaky_relu(x + b.reshape(1, -1, 1, 1), 0.2)

    def run(self, image: np.ndarray) -> dict:
        """image [3, 512, 512] -> appearance [512], lambda [20], motion [512],
        feats[j] [r*r, C] channel-last (menc conv{6-j})"""
        p = "enc.net_app.convs."
        x = self._flrelu(self._conv(_t(image)[None], p + "0.0.weight"), self.w[p + "0.1.bias"])
        pyr = [x]
        for i in range(1, 8):
            b = f"{p}{i}."
            h = self._flrelu(self._conv(x, b + "conv1.0.weight", pad=1), self.w[b + "conv1.1.bias"])
            h = _upfirdn(h, self.w[b + "conv2.0.kernel"], 1, 2, 2)
            h = self._flrelu(self._conv(h, b + "conv2.1.weight", stride=2), self.w[b + "conv2.2.bias"])
            s = _upfirdn(x, self.w[b + "skip.0.kernel"], 1, 1, 1)
            s = self._conv(s, b + "skip.1.weight", stride=2)
            x = (h + s) / math.sqrt(2.0)
            pyr.append(x)
        app = self._conv(x, p + "8.weight")[0, :, 0, 0]
        h = app
        for i in range(5):
            W = self.w[f"enc.fc.{i}.weight"]
            h = h @ (W * (1.0 / math.sqrt(W.shape[1]))).T + self.w[f"enc.fc.{i}.bias"]
        motion = self.w["dec.direction.Q"] @ h
        feats = []
        for j in range(7):
            f = pyr[6 - j][0]
            feats.append(f.reshape(f.shape[0], -1).T.numpy())
        return dict(appearance=app.numpy(), lam=h.numpy(), motion=motion.numpy(), feats=feats)


class TorchFmt:
    """The flow-matching DiT forward in float64 torch, written from the
    module definitions (DiT blocks with adaLN modulation h*(1+scale)+shift,
    LayerNorm without affine, tanh GELU, banded attention |i-j| <= window via
    an additive -inf mask, SiLU conditioning), independent of the oracle."""

    def __init__(self, cfg: dict, raw: dict):
        self.c = cfg
        self.w = {k: _t(v) for k, v in raw.items()}

    def _lin(self, n, x):
        return x @ self.w[n + ".weight"].T + self.w[n + ".bias"]

    def forward(self, x60, cond, t: float) -> np.ndarray:
        c = self.c
        H, T, nh = c["dim_h"], c["chunk_frames"] + c["prev_frames"], c["n_heads"]
        hd = H // nh
        half = c["t_freq_dim"] // 2
        fr = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
        tf = torch.cat([torch.cos(t * fr), torch.sin(t * fr)])
        te = self._lin("t_embedder.mlp.2", F.silu(self._lin("t_embedder.mlp.0", tf)))
        sc = F.silu(self._lin("c_embedder", _t(cond)) + te)          # [3, T, H]
        x = (self._lin("x_embedder.proj", _t(x60)) + self.w["pos_embed"][0])[None].repeat(3, 1, 1)
        i = torch.arange(T)
        mask = torch.where((i[:, None] - i[None, :]).abs() <= c["attn_window"], 0.0, -math.inf)
        ln = lambda z: F.layer_norm(z, (H,), eps=c["ln_eps"])
        for l in range(c["depth"]):
            b = f"blocks.{l}."
            sh1, sc1, g1, sh2, sc2, g2 = self._lin(b + "adaLN_modulation.1", sc).chunk(6, -1)
            h = ln(x) * (1 + sc1) + sh1
            q, k, v = self._lin(b + "attn.qkv", h).chunk(3, -1)
            q, k, v = [z.reshape(3, T, nh, hd).transpose(1, 2) for z in (q, k, v)]
            a = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(hd) + mask, -1) @ v
            a = a.transpose(1, 2).reshape(3, T, H)
            x = x + g1 * self._lin(b + "attn.proj", a)
            h = ln(x) * (1 + sc2) + sh2
            x = x + g2 * self._lin(b + "mlp.fc2", F.gelu(self._lin(b + "mlp.fc1", h), approximate="tanh"))
        shf, scf = self._lin("decoder.adaLN_modulation.1", sc).chunk(2, -1)
        return self._lin("decoder.linear", ln(x) * (1 + scf) + shf).numpy()


class TorchAudio:
    """The modified wav2vec2 audio encoder in float64 torch (conv1d stem with
    a per-channel GroupNorm, exact-erf GELU, align_corners linear
    interpolation, grouped positional conv, post-norm transformer layers,
    projection of all layer outputs), independent of the oracle."""

    def __init__(self, cfg: dict, raw: dict):
        self.c = cfg
        self.w = {k: _t(v) for k, v in raw.items()}

    def encode(self, audio: np.ndarray, seq_len: int) -> np.ndarray:
        c, w = self.c, self.w
        x = _t(audio)
        unit = seq_len * c["sample_rate"] // c["fps"]
        if unit > 0 and x.numel() % unit != 0:
            pad = torch.full((unit,), float(x[-1]), dtype=torch.float64)
            m = min(unit, x.numel())
            pad[:m] = x[:m]
            x = pad
        h = x[None, None]
        for i in range(7):
            h = F.conv1d(h, w[f"feature_extractor.conv_layers.{i}.conv.weight"], stride=c["conv_stride"][i])
            if i == 0:
                h = F.group_norm(h, h.shape[1], w["feature_extractor.conv_layers.0.layer_norm.weight"],
                                 w["feature_extractor.conv_layers.0.layer_norm.bias"], eps=c["ln_eps"])
            h = F.gelu(h)
        h = F.interpolate(h, size=seq_len, mode="linear", align_corners=True)[0].T   # [S, C]
        h = F.layer_norm(h, (h.shape[1],), w["feature_projection.layer_norm.weight"],
                         w["feature_projection.layer_norm.bias"], eps=c["ln_eps"])
        h = h @ w["feature_projection.projection.weight"].T + w["feature_projection.projection.bias"]
        K = c["pos_kernel"]
        pos = F.conv1d(h.T[None], w["encoder.pos_conv_embed.conv.weight"], w["encoder.pos_conv_embed.conv.bias"],
                       padding=K // 2, groups=c["pos_groups"])[0, :, :seq_len]
        h = h + F.gelu(pos).T
        Hd, nh = c["hidden"], c["n_heads"]
        ln = lambda z, n: F.layer_norm(z, (Hd,), w[n + ".weight"], w[n + ".bias"], eps=c["ln_eps"])
        h = ln(h, "encoder.layer_norm")
        outs = []
        for l in range(c["n_layers"]):
            b = f"encoder.layers.{l}."
            lin = lambda z, n: z @ w[b + n + ".weight"].T + w[b + n + ".bias"]
            q = lin(h, "attention.q_proj") / math.sqrt(Hd // nh)
            k, v = lin(h, "attention.k_proj"), lin(h, "attention.v_proj")
            q, k, v = [z.reshape(seq_len, nh, -1).transpose(0, 1) for z in (q, k, v)]
            a = (torch.softmax(q @ k.transpose(-1, -2), -1) @ v).transpose(0, 1).reshape(seq_len, Hd)
            h = ln(h + lin(a, "attention.out_proj"), b + "layer_norm")
            f = lin(F.gelu(lin(h, "feed_forward.intermediate_dense")), "feed_forward.output_dense")
            h = ln(h + f, b + "final_layer_norm")
            outs.append(h)
        st = torch.cat(outs, -1)
        o = st @ w["audio_projection.0.weight"].T + w["audio_projection.0.bias"]
        o = F.layer_norm(o, (c["dim_w"],), w["audio_projection.1.weight"], w["audio_projection.1.bias"], eps=1e-5)
        return F.silu(o).numpy()
