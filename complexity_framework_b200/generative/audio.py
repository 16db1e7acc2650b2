"""Audio: log-mel front end, TR-Hash audio encoder, speech-to-text and
text-to-speech.

Counterparts: complexity/generative/audio/ (mel.py ``build_mel_filterbank`` /
``LogMelSpectrogram``, encoder.py ``AudioEncoder`` / ``AudioEncoderConfig``,
model.py ``TokenResampler``, ``TRHashSpeechToText``, ``TRHashTextToSpeech``,
config.py).  The filter bank is the usual triangular bank on the HTK mel scale
(2595 log10(1 + f/700)); frames route through the TR-Hash experts by frame
position.  Text-to-speech predicts mel frames from the decoder's hidden
states upsampled by a fixed number of frames per token (L1 loss); a vocoder
is outside this package.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .prefix_lm import PrefixLM, TokenResampler
from .towers import TRHashVisionBlock


def _hz_to_mel(f):
    return 2595.0 * torch.log10(1.0 + f / 700.0)


def _mel_to_hz(m):
    return 700.0 * (10.0 ** (m / 2595.0) - 1.0)


def build_mel_filterbank(n_mels: int, n_fft: int, sample_rate: int, f_min: float = 0.0,
                         f_max: Optional[float] = None) -> torch.Tensor:
    """[n_mels, n_fft // 2 + 1] triangular filters, peaks evenly spaced in mel."""
    f_max = sample_rate / 2 if f_max is None else f_max
    freqs = torch.linspace(0, sample_rate / 2, n_fft // 2 + 1, dtype=torch.float64)
    pts = _mel_to_hz(torch.linspace(float(_hz_to_mel(torch.tensor(f_min))),
                                    float(_hz_to_mel(torch.tensor(f_max))), n_mels + 2,
                                    dtype=torch.float64))
    lo, ctr, hi = pts[:-2, None], pts[1:-1, None], pts[2:, None]
    up = (freqs[None] - lo) / (ctr - lo)
    down = (hi - freqs[None]) / (hi - ctr)
    return torch.clamp(torch.minimum(up, down), min=0.0).float()


class LogMelSpectrogram(nn.Module):
    """[B, samples] waveform -> [B, n_mels, frames] log10 mel power (floored)."""

    def __init__(self, sample_rate: int = 16000, n_fft: int = 400, hop_length: int = 160,
                 n_mels: int = 80, floor: float = 1e-10):
        super().__init__()
        self.n_fft, self.hop, self.floor = n_fft, hop_length, floor
        self.register_buffer("window", torch.hann_window(n_fft), persistent=False)
        self.register_buffer("fb", build_mel_filterbank(n_mels, n_fft, sample_rate),
                             persistent=False)

    def forward(self, audio: torch.Tensor) -> torch.Tensor:
        spec = torch.stft(audio.float(), self.n_fft, self.hop, window=self.window,
                          return_complex=True).abs() ** 2
        return torch.log10((self.fb @ spec).clamp_min(self.floor))


@dataclass
class AudioEncoderConfig:
    n_mels: int = 80
    max_frames: int = 3000          # mel frames (30 s at 10 ms hop); encoder keeps half
    hidden_size: int = 384
    num_layers: int = 4
    num_heads: int = 6
    num_experts: int = 4
    top_k: int = 2
    shared_width: int = 768
    expert_width: int = 128
    dropout: float = 0.0
    route_seed: int = 0xA0D10

    @property
    def route_vocab_size(self) -> int:
        return self.max_frames // 2 + 1


class AudioEncoder(nn.Module):
    """Two convolutions (the second strided by 2) then TR-Hash blocks keyed on
    frame position: [B, n_mels, frames] -> [B, ceil(frames / 2), hidden]."""

    def __init__(self, config: AudioEncoderConfig):
        super().__init__()
        self.config = c = config
        self.conv1 = nn.Conv1d(c.n_mels, c.hidden_size, 3, padding=1)
        self.conv2 = nn.Conv1d(c.hidden_size, c.hidden_size, 3, stride=2, padding=1)
        self.pos = nn.Parameter(torch.randn(1, c.route_vocab_size, c.hidden_size) * 0.02)
        self.blocks = nn.ModuleList(TRHashVisionBlock(c, i) for i in range(c.num_layers))
        self.norm = nn.LayerNorm(c.hidden_size)

    def forward(self, mel: torch.Tensor) -> torch.Tensor:
        x = F.gelu(self.conv2(F.gelu(self.conv1(mel)))).transpose(1, 2)
        n = x.shape[1]
        if n > self.pos.shape[1]:
            raise ValueError(f"{n} encoder frames exceed max_frames // 2 + 1")
        x = x + self.pos[:, :n].to(x.dtype)
        ids = torch.arange(n, device=x.device).unsqueeze(0).expand(x.shape[0], -1)
        for b in self.blocks:
            x = b(x, ids)
        return self.norm(x)


@dataclass
class TRHashAudioConfig:
    sample_rate: int = 16000
    n_fft: int = 400
    hop_length: int = 160
    encoder: AudioEncoderConfig = None
    num_audio_tokens: int = 32        # resampled prefix length (speech-to-text)
    frames_per_token: int = 4         # text-to-speech upsampling

    def __post_init__(self):
        if self.encoder is None:
            self.encoder = AudioEncoderConfig()


TRHashSpeechToTextConfig = TRHashAudioConfig


class TRHashSpeechToText(nn.Module):
    """Waveform (or mel) -> text: audio encoder, token resampler, TR-Hash decoder."""

    def __init__(self, config: TRHashAudioConfig, decoder):
        super().__init__()
        self.config = config
        e = config.encoder
        self.mel = LogMelSpectrogram(config.sample_rate, config.n_fft, config.hop_length, e.n_mels)
        self.encoder = AudioEncoder(e)
        self.resampler = TokenResampler(e.hidden_size, decoder.config.hidden_size,
                                        config.num_audio_tokens, max(1, e.num_heads // 2))
        self.lm = PrefixLM(decoder)

    def prefix(self, audio: Optional[torch.Tensor] = None,
               mel: Optional[torch.Tensor] = None) -> torch.Tensor:
        if mel is None:
            mel = self.mel(audio)
        return self.resampler(self.encoder(mel))

    def forward(self, input_ids: torch.Tensor, audio: Optional[torch.Tensor] = None,
                mel: Optional[torch.Tensor] = None, labels: Optional[torch.Tensor] = None) -> dict:
        return {"loss": self.lm.loss(self.prefix(audio, mel), input_ids, labels)}

    def transcribe(self, audio: torch.Tensor, bos_id: int, max_new_tokens: int = 64,
                   eos_id: Optional[int] = None) -> torch.Tensor:
        bos = torch.full((audio.shape[0], 1), bos_id, dtype=torch.long, device=audio.device)
        return self.lm.generate(self.prefix(audio), bos, max_new_tokens, eos_id)


class TRHashTextToSpeech(nn.Module):
    """Text -> mel frames: decoder hidden states, upsampled ``frames_per_token``
    times (repeat + learned offset per sub-frame), TR-Hash blocks over frames,
    linear to mel bins.  Trained with L1 against target mels."""

    def __init__(self, config: TRHashAudioConfig, decoder):
        super().__init__()
        self.config = config
        e = config.encoder
        self.decoder = decoder
        H = decoder.config.hidden_size
        self.in_proj = nn.Linear(H, e.hidden_size)
        self.sub = nn.Parameter(torch.zeros(config.frames_per_token, e.hidden_size))
        self.blocks = nn.ModuleList(TRHashVisionBlock(e, i) for i in range(e.num_layers))
        self.norm = nn.LayerNorm(e.hidden_size)
        self.out = nn.Linear(e.hidden_size, e.n_mels)

    def forward(self, input_ids: torch.Tensor, mel: Optional[torch.Tensor] = None) -> dict:
        h = self.decoder(input_ids, return_logits=False)["last_hidden_state"]
        x = self.in_proj(h)
        B, T, D = x.shape
        k = self.config.frames_per_token
        x = (x[:, :, None, :] + self.sub.to(x.dtype)).reshape(B, T * k, D)
        n = x.shape[1]
        vocab = self.config.encoder.route_vocab_size
        ids = (torch.arange(n, device=x.device) % vocab).unsqueeze(0).expand(B, -1)
        for b in self.blocks:
            x = b(x, ids)
        pred = self.out(self.norm(x)).transpose(1, 2)     # [B, n_mels, T * k]
        out = {"mel": pred}
        if mel is not None:
            m = min(mel.shape[-1], pred.shape[-1])
            out["loss"] = F.l1_loss(pred[..., :m].float(), mel[..., :m].float())
        return out
