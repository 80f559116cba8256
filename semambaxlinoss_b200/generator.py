"""SEMamba generator harness for the generator-level workloads (training step, long
inference) — the measurement harness around this package's TF-blocks.

The parts of the generator that are not scans are restated in plain PyTorch (cuDNN
convolutions, cuFFT STFT) from the reference, unoptimised; they are the harness, not the
hot path:

* ``DenseBlock`` / ``DenseEncoder`` / ``MagDecoder`` / ``PhaseDecoder`` /
  ``LearnableSigmoid2D``: reference models/codec_module.py:35-69, 139-269 and
  models/lsigmoid.py (the FAN variants are not included);
* ``SEMamba``: reference models/generator.py:7-77;
* ``mag_phase_stft`` / ``mag_phase_istft``: reference models/stfts.py:4-73;
* ``generator_loss``: the generator terms of the reference training step
  (train.py:603-624: magnitude L2, anti-wrapping phase losses, complex L2, time L1,
  STFT consistency; models/loss.py:9-60), without the discriminator / PESQ metric term.

``config3_cfg()`` is the generator of the training-step workload: 64 hidden channels, 4
TF-blocks, time axis = selective-LRU (d_inner 256, 16 modes, conv 4, gamma gain),
frequency axis = damped-IMEX LinOSS (16 oscillators), bidirectional.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .mamba_block import TFMambaBlock


def config3_cfg(num_tfmamba: int = 4) -> dict:
    mixer = dict(d_conv=4, expand=4, norm_epsilon=1e-5, causal_conv=True, bidirectional=True)
    return {
        "stft_cfg": dict(sampling_rate=16000, n_fft=400, hop_size=100, win_size=400),
        "model_cfg": dict(
            hid_feature=64, dense_stride=2, compress_factor=0.3, num_tfmamba=num_tfmamba, beta=2.0,
            input_channel=2, output_channel=1, use_transpose=True,
            time_mixer=dict(mixer, ssm="selective_lru", d_state=16,
                            ssm_params=dict(input_gain="gamma", chunk_size=16)),
            freq_mixer=dict(mixer, ssm="linoss", d_state=16,
                            ssm_params=dict(discretization="IMEX", damping=True)),
        ),
        "training_cfg": dict(loss=dict(magnitude=0.9, phase=0.3, complex=0.1, time=0.2, consistancy=0.1)),
    }


def _pad2d(kernel, dilation=(1, 1)):
    return ((kernel[0] * dilation[0] - dilation[0]) // 2, (kernel[1] * dilation[1] - dilation[1]) // 2)


class LearnableSigmoid2D(nn.Module):
    """beta * sigmoid(slope * x) with a learned per-bin slope (in_features, 1)."""

    def __init__(self, in_features, beta=1.0):
        super().__init__()
        self.beta = beta
        self.slope = nn.Parameter(torch.ones(in_features, 1))

    def forward(self, x):
        return self.beta * torch.sigmoid(self.slope * x)


class DenseBlock(nn.Module):
    """``depth`` dilated 3x3 conv -> InstanceNorm -> PReLU layers with dense concatenation
    of all previous outputs; dilation 2^i along time."""

    def __init__(self, cfg, kernel_size=(3, 3), depth=4):
        super().__init__()
        hid = cfg["model_cfg"]["hid_feature"]
        self.depth = depth
        self.dense_block = nn.ModuleList(
            nn.Sequential(
                nn.Conv2d(hid * (i + 1), hid, kernel_size, dilation=(2**i, 1),
                          padding=_pad2d(kernel_size, (2**i, 1))),
                nn.InstanceNorm2d(hid, affine=True),
                nn.PReLU(hid),
            )
            for i in range(depth)
        )

    def forward(self, x):
        skip = x
        for i in range(self.depth):
            x = self.dense_block[i](skip)
            skip = torch.cat([x, skip], dim=1)
        return x


class DenseEncoder(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        mc = cfg["model_cfg"]
        hid, stride = mc["hid_feature"], mc.get("dense_stride", 2)
        self.dense_conv_1 = nn.Sequential(nn.Conv2d(mc["input_channel"], hid, (1, 1)),
                                          nn.InstanceNorm2d(hid, affine=True), nn.PReLU(hid))
        self.dense_block = DenseBlock(cfg, depth=4)
        self.dense_conv_2 = nn.Sequential(nn.Conv2d(hid, hid, (1, 3), stride=(1, stride)),
                                          nn.InstanceNorm2d(hid, affine=True), nn.PReLU(hid))

    def forward(self, x):
        return self.dense_conv_2(self.dense_block(self.dense_conv_1(x)))


class MagDecoder(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        mc = cfg["model_cfg"]
        hid, out, stride = mc["hid_feature"], mc["output_channel"], mc.get("dense_stride", 2)
        self.dense_block = DenseBlock(cfg, depth=4)
        self.mask_conv = nn.Sequential(
            nn.ConvTranspose2d(hid, hid, (1, 3), stride=(1, stride)),
            nn.Conv2d(hid, out, (1, 1)),
            nn.InstanceNorm2d(out, affine=True),
            nn.PReLU(out),
            nn.Conv2d(out, out, (1, 1)),
        )
        self.lsigmoid = LearnableSigmoid2D(cfg["stft_cfg"]["n_fft"] // 2 + 1, beta=mc["beta"])

    def forward(self, x):
        x = self.mask_conv(self.dense_block(x))          # (b, 1, t, f)
        x = self.lsigmoid(x.permute(0, 3, 2, 1).squeeze(-1))  # (b, f, t)
        return x.transpose(1, 2).unsqueeze(1)             # (b, 1, t, f)


class PhaseDecoder(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        mc = cfg["model_cfg"]
        hid, out, stride = mc["hid_feature"], mc["output_channel"], mc.get("dense_stride", 2)
        self.dense_block = DenseBlock(cfg, depth=4)
        self.phase_conv = nn.Sequential(nn.ConvTranspose2d(hid, hid, (1, 3), stride=(1, stride)),
                                        nn.InstanceNorm2d(hid, affine=True), nn.PReLU(hid))
        self.phase_conv_r = nn.Conv2d(hid, out, (1, 1))
        self.phase_conv_i = nn.Conv2d(hid, out, (1, 1))

    def forward(self, x):
        x = self.phase_conv(self.dense_block(x))
        return torch.atan2(self.phase_conv_i(x), self.phase_conv_r(x))


class SEMamba(nn.Module):
    """noisy (mag, pha) [B, F, T] -> (mag, pha, complex [B, F, T, 2])."""

    def __init__(self, cfg):
        super().__init__()
        n = cfg["model_cfg"].get("num_tfmamba") or 4
        self.dense_encoder = DenseEncoder(cfg)
        self.TSMamba = nn.ModuleList(TFMambaBlock(cfg, layer_idx=i, num_layers=n) for i in range(n))
        self.mask_decoder = MagDecoder(cfg)
        self.phase_decoder = PhaseDecoder(cfg)

    def forward(self, noisy_mag, noisy_pha):
        mag = noisy_mag.transpose(1, 2).unsqueeze(1)  # (b, 1, t, f)
        pha = noisy_pha.transpose(1, 2).unsqueeze(1)
        x = self.dense_encoder(torch.cat((mag, pha), dim=1))
        for block in self.TSMamba:
            x = block(x)
        den_mag = (self.mask_decoder(x) * mag).permute(0, 3, 2, 1).squeeze(-1)
        den_pha = self.phase_decoder(x).permute(0, 3, 2, 1).squeeze(-1)
        den_com = torch.stack((den_mag * torch.cos(den_pha), den_mag * torch.sin(den_pha)), dim=-1)
        return den_mag, den_pha, den_com


def mag_phase_stft(y, n_fft, hop_size, win_size, compress_factor=1.0, center=True, addeps=False):
    window = torch.hann_window(win_size, device=y.device)
    spec = torch.stft(y, n_fft, hop_length=hop_size, win_length=win_size, window=window, center=center,
                      pad_mode="reflect", normalized=False, return_complex=True)
    if addeps:
        eps = 1e-10
        mag = torch.sqrt(spec.real.pow(2) + spec.imag.pow(2) + eps)
        pha = torch.atan2(spec.imag + eps, spec.real + eps)
    else:
        mag, pha = torch.abs(spec), torch.angle(spec)
    mag = torch.pow(mag, compress_factor)
    com = torch.stack((mag * torch.cos(pha), mag * torch.sin(pha)), dim=-1)
    return mag, pha, com


def mag_phase_istft(mag, pha, n_fft, hop_size, win_size, compress_factor=1.0, center=True):
    mag = torch.pow(mag, 1.0 / compress_factor)
    com = torch.complex(mag * torch.cos(pha), mag * torch.sin(pha))
    window = torch.hann_window(win_size, device=com.device)
    return torch.istft(com, n_fft, hop_length=hop_size, win_length=win_size, window=window, center=center)


def _anti_wrap(x):
    return torch.abs(x - torch.round(x / (2 * math.pi)) * 2 * math.pi)


def _delay_matrix(n, device):
    """(n, n) matrix D with D[i, i] = -1, D[i, i+1] = 1: x @ D gives x[j-1] - x[j]."""
    return (torch.triu(torch.ones(n, n, device=device), 1) - torch.triu(torch.ones(n, n, device=device), 2)
            - torch.eye(n, device=device))


def phase_losses(phase_r, phase_g):
    """In-phase, group-delay and instantaneous-frequency anti-wrapping losses."""
    gd = _delay_matrix(phase_r.size(1), phase_r.device)
    iaf = _delay_matrix(phase_r.size(-1), phase_r.device)
    ip = torch.mean(_anti_wrap(phase_r - phase_g))
    gdl = torch.mean(_anti_wrap(phase_r.transpose(1, 2) @ gd - phase_g.transpose(1, 2) @ gd))
    iafl = torch.mean(_anti_wrap(phase_r @ iaf - phase_g @ iaf))
    return ip, gdl, iafl


def generator_loss(cfg, clean_audio, clean_mag, clean_pha, clean_com, mag_g, pha_g, com_g):
    sc, w = cfg["stft_cfg"], cfg["training_cfg"]["loss"]
    cf = cfg["model_cfg"]["compress_factor"]
    audio_g = mag_phase_istft(mag_g, pha_g, sc["n_fft"], sc["hop_size"], sc["win_size"], cf)
    loss_mag = F.mse_loss(clean_mag, mag_g)
    loss_pha = sum(phase_losses(clean_pha, pha_g))
    loss_com = F.mse_loss(clean_com, com_g)
    loss_time = F.l1_loss(clean_audio, audio_g)
    _, _, rec_com = mag_phase_stft(audio_g, sc["n_fft"], sc["hop_size"], sc["win_size"], cf, addeps=True)
    loss_con = F.mse_loss(com_g, rec_com)
    return (loss_mag * w["magnitude"] + loss_pha * w["phase"] + loss_com * 2 * w["complex"]
            + loss_time * w["time"] + loss_con * 2 * w["consistancy"])
