"""MiniMax-H3 packed-sequence layout: row order, modality tags and 3-axis rotary positions.

The model sees ONE packed sequence [text | keyframe-condition video | audio | video]
with per-row (t, h, w) rotary coordinates.  The numbers are the released model's
contract (difflet/models/minimax_h3/contracts.py:17-353) and must match it exactly
for the released weights to work: 24 fps, 40 audio latents per second over 2
channels, 16x spatial VAE compression with (1, 2, 2) patches, 17 n + 5 frames ->
5 n + 2 latent frames, rotary time spans (1, 4, 4, 4, 4) x 5/3 per latent frame
starting after the text, spatial positions centred on the canvas and scaled by 32,
audio rows at the text-following times with the two channels at the first / last
width position, keyframe blocks at the first / last latent frame time.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

VIDEO_TAG, TEXT_TAG, AUDIO_TAG = 0, 1, 2
FPS = 24
AUDIO_LATENTS_PER_SECOND = 40
AUDIO_CHANNELS = 2
VAE_SPATIAL = 16
PATCH = (1, 2, 2)
FRAMES_PER_CHUNK, LATENTS_PER_CHUNK = 17, 5
KEYFRAME_NOISE_AUG = 0.999
_FRAME_RESCALE = 5.0 / 3.0
_FRAMES_PER_LATENT = (1, 4, 4, 4, 4)
_SPATIAL_SCALE = 32


@dataclass(frozen=True)
class Layout:
    num_latent_frames: int
    num_audio_latents: int
    position_ids: torch.Tensor   # [S, 3] float64
    token_tags: torch.Tensor     # [S] int64
    video_indices: torch.Tensor
    audio_indices: torch.Tensor
    text_indices: torch.Tensor
    num_condition_rows: int = 0

    @property
    def sequence_length(self) -> int:
        return int(self.position_ids.shape[0])


def align_num_frames(n: int) -> int:
    while n % FRAMES_PER_CHUNK != LATENTS_PER_CHUNK:
        n += 1
    return n


def video_latent_frames(num_frames: int) -> int:
    if num_frames % FRAMES_PER_CHUNK != LATENTS_PER_CHUNK:
        raise ValueError(f"num_frames must be 17 n + 5, got {num_frames}")
    return (num_frames - LATENTS_PER_CHUNK) // FRAMES_PER_CHUNK * LATENTS_PER_CHUNK + 2


def audio_latent_frames(num_frames: int) -> int:
    return int(round(num_frames / FPS * AUDIO_LATENTS_PER_SECOND))


def _spatial_grid(n: int, patch: int, sqrt_area: float) -> torch.Tensor:
    ratio = n / sqrt_area
    left = (1.0 - ratio) / 2.0
    return torch.from_numpy(np.linspace(left, left + ratio, n // patch, endpoint=False) * _SPATIAL_SCALE)


def _frame_grid(lh: int, lw: int):
    sq = float(np.sqrt(lh * lw))
    hg, wg = _spatial_grid(lh, PATCH[1], sq), _spatial_grid(lw, PATCH[2], sq)
    gh, gw = torch.meshgrid(hg, wg, indexing="ij")
    return torch.stack([gh.reshape(-1), gw.reshape(-1)], -1), wg


def _time_grid(nf: int, origin: float) -> torch.Tensor:
    spans = torch.tensor([_FRAME_RESCALE * _FRAMES_PER_LATENT[i % len(_FRAMES_PER_LATENT)] for i in range(nf)],
                         dtype=torch.float64)
    return origin + torch.cat([torch.zeros(1, dtype=torch.float64), spans[:-1].cumsum(0)])


def keyframe_time(anchor: str, num_text: int, nf: int) -> float:
    if anchor == "first":
        return float(num_text)
    if anchor == "last":
        spans = np.ones(nf, dtype=np.float64) * _FRAME_RESCALE
        for o in range(len(_FRAMES_PER_LATENT)):
            spans[o::len(_FRAMES_PER_LATENT)] *= _FRAMES_PER_LATENT[o]
        return float(num_text) + float(spans.sum()) - _FRAME_RESCALE
    raise ValueError(f"keyframe anchor must be 'first' or 'last', got {anchor!r}")


def build_layout(*, num_text_tokens: int, height: int, width: int, num_frames: int,
                 keyframe_anchors: tuple = (), check_duration: bool = True) -> Layout:
    if num_text_tokens < 1:
        raise ValueError("MiniMax-H3 needs at least one text token")
    if height % 32 or width % 32:
        raise ValueError(f"height and width must be multiples of 32, got {height}x{width}")
    if check_duration and not 120 <= num_frames <= 360:
        raise ValueError(f"MiniMax-H3 generates 5-15 seconds at 24 fps, got {num_frames} frames")
    lh, lw = height // VAE_SPATIAL, width // VAE_SPATIAL
    rows_per_frame = (lh // PATCH[1]) * (lw // PATCH[2])
    nf = video_latent_frames(num_frames)
    na = audio_latent_frames(num_frames)
    n_audio, n_video = na * AUDIO_CHANNELS, nf * rows_per_frame
    n_cond = len(keyframe_anchors) * rows_per_frame
    S = num_text_tokens + n_cond + n_audio + n_video
    c0 = num_text_tokens
    a0 = c0 + n_cond
    v0 = a0 + n_audio
    pos = torch.zeros(S, 3, dtype=torch.float64)
    pos[:num_text_tokens, 0] = torch.arange(num_text_tokens, dtype=torch.float64)
    fg, wg = _frame_grid(lh, lw)
    for i, anchor in enumerate(keyframe_anchors):
        rows = slice(c0 + i * rows_per_frame, c0 + (i + 1) * rows_per_frame)
        pos[rows, 0] = keyframe_time(anchor, num_text_tokens, nf)
        pos[rows, 1:] = fg
    at = float(num_text_tokens) + torch.arange(na, dtype=torch.float64)
    pos[a0:v0, 0] = at.repeat(AUDIO_CHANNELS)
    pos[a0:v0, 2] = torch.cat([torch.full((na,), float(wg[0]), dtype=torch.float64),
                               torch.full((na,), float(wg[-1]), dtype=torch.float64)])
    vp = torch.empty(nf, rows_per_frame, 3, dtype=torch.float64)
    vp[:, :, 0] = _time_grid(nf, float(num_text_tokens))[:, None]
    vp[:, :, 1:] = fg[None]
    pos[v0:] = vp.reshape(-1, 3)
    text_idx = torch.arange(num_text_tokens)
    audio_idx = torch.arange(a0, v0)
    video_idx = torch.cat([torch.arange(c0, a0), torch.arange(v0, S)])
    tags = torch.empty(S, dtype=torch.long)
    tags[text_idx] = TEXT_TAG
    tags[audio_idx] = AUDIO_TAG
    tags[video_idx] = VIDEO_TAG
    return Layout(nf, na, pos, tags, video_idx, audio_idx, text_idx, n_cond)


def patchify(lat: torch.Tensor) -> torch.Tensor:
    """[B, C, F, H, W] -> [B, F (H/2) (W/2), C * 1 * 2 * 2] rows (patch (1, 2, 2), channel-major)."""
    B, C, Fr, H, W = lat.shape
    x = lat.view(B, C, Fr, H // 2, 2, W // 2, 2).permute(0, 2, 3, 5, 1, 4, 6)
    return x.reshape(B, Fr * (H // 2) * (W // 2), C * 4)


def unpatchify(rows: torch.Tensor, channels: int, nf: int, lh: int, lw: int) -> torch.Tensor:
    B = rows.shape[0]
    x = rows.view(B, nf, lh // 2, lw // 2, channels, 2, 2).permute(0, 4, 1, 2, 5, 3, 6)
    return x.reshape(B, channels, nf, lh, lw)


__all__ = ["AUDIO_CHANNELS", "AUDIO_TAG", "KEYFRAME_NOISE_AUG", "Layout", "TEXT_TAG", "VIDEO_TAG", "align_num_frames",
           "audio_latent_frames", "build_layout", "keyframe_time", "patchify", "unpatchify", "video_latent_frames"]
