"""Speech-to-text front end of the audio cascade.

The decoder never sees audio: each clip is transcribed and its transcript
spliced into the prompt as text tokens (reference: src/granite_switch/vllm/audio/asr.py:285-560).
:class:`ASRTranscriber` normalises a clip (``(array, rate)`` or array plus
``sampling_rate``; numpy, list or torch; downmixed to mono float32),
resamples it to 16 kHz with a polyphase filter, and either hands the whole
clip to the backend (``self_chunks=True``, for backends that window on their
own) or cuts it into overlapping windows and merges the window transcripts
(:mod:`.chunking`).

The backend is any callable ``(samples_16k: np.ndarray) -> str``. By default it
is a lazily built ``transformers`` speech-recognition pipeline for
``model_id`` (CTC models decode in one pass; generative ones get
``generate_kwargs`` and their own 30 s windowing). Transcribers are cached
per (model, revision, device, dtype, pipeline kwargs).
"""
from __future__ import annotations

import math
import threading
from typing import Any, Callable, Mapping

import numpy as np

from .chunking import merge_transcripts, split_waveform

TARGET_SAMPLE_RATE = 16_000
SEQ2SEQ_WINDOW_S = 30.0
# request-level generate kwargs a client may set; the rest come from the checkpoint config
ALLOWED_REQUEST_GENERATE_KEYS = frozenset({"language", "task"})


def to_mono_float32(samples) -> np.ndarray:
    if hasattr(samples, "detach") and hasattr(samples, "cpu"):
        samples = samples.detach().cpu().numpy()
    a = np.asarray(samples)
    if a.ndim > 1:  # channels on the shorter axis
        a = a.mean(axis=int(np.argmin(a.shape)))
    return a.astype(np.float32, copy=False)


def resample(samples: np.ndarray, orig_sr: int, target_sr: int = TARGET_SAMPLE_RATE) -> np.ndarray:
    """Polyphase resampling (scipy.signal.resample_poly) by the reduced ratio target/orig."""
    if orig_sr == target_sr:
        return samples
    if orig_sr <= 0:
        raise ValueError(f"sampling rate must be positive, got {orig_sr}")
    from scipy.signal import resample_poly

    g = math.gcd(int(target_sr), int(orig_sr))
    return resample_poly(samples, int(target_sr) // g, int(orig_sr) // g).astype(np.float32)


def coerce_audio(audio, sampling_rate: int | None) -> tuple[np.ndarray, int]:
    if isinstance(audio, tuple):
        if len(audio) != 2:
            raise ValueError(f"tuple audio input must be (array, sampling_rate); got length {len(audio)}")
        return to_mono_float32(audio[0]), int(audio[1])
    if sampling_rate is None:
        raise ValueError("sampling_rate is required when audio is not an (array, sampling_rate) tuple")
    return to_mono_float32(audio), int(sampling_rate)


def resolve_generate_kwargs(config_defaults: Mapping[str, Any] | None, request: Mapping[str, Any] | None = None,
                            allowed: frozenset = ALLOWED_REQUEST_GENERATE_KEYS) -> dict[str, Any]:
    """Checkpoint defaults overlaid with the request's allow-listed keys; others are refused."""
    out = dict(config_defaults or {})
    for k, v in (request or {}).items():
        if k not in allowed:
            raise ValueError(f"generate kwarg {k!r} may not be set per request (allowed: {sorted(allowed)})")
        out[k] = v
    return out


class ASRTranscriber:
    def __init__(self, model_id: str | None = None, device: str = "cuda", dtype: str | None = None,
                 revision: str | None = None, pipeline_kwargs: Mapping[str, Any] | None = None,
                 backend: Callable[[np.ndarray], str] | None = None):
        self.model_id, self.device, self.dtype, self.revision = model_id, device, dtype, revision
        self.pipeline_kwargs = dict(pipeline_kwargs or {})
        self._backend = backend
        self._pipe = None
        self._ctc = False
        self._lock = threading.Lock()

    def _build_pipeline(self):
        with self._lock:
            if self._pipe is not None:
                return
            from transformers import pipeline  # lazy: the rest imports without the audio stack

            import torch

            kw: dict[str, Any] = dict(task="automatic-speech-recognition", model=self.model_id, device=self.device)
            if self.dtype:
                kw["torch_dtype"] = getattr(torch, self.dtype)
            if self.revision is not None:
                kw["revision"] = self.revision
            kw.update(self.pipeline_kwargs)
            self._pipe = pipeline(**kw)
            self._ctc = getattr(self._pipe, "type", None) == "ctc" or "ctc" in type(self._pipe.model).__name__.lower()

    def _run(self, samples: np.ndarray, generate_kwargs: Mapping[str, Any] | None) -> str:
        if self._backend is not None:
            return str(self._backend(samples)).strip()
        if self.model_id is None:
            raise ValueError("no ASR model configured (asr_model_id / asr_bundled_path) and no backend given")
        self._build_pipeline()
        call: dict[str, Any] = {}
        if not self._ctc:
            if generate_kwargs:
                call["generate_kwargs"] = dict(generate_kwargs)
            if "chunk_length_s" not in self.pipeline_kwargs:
                call["chunk_length_s"] = SEQ2SEQ_WINDOW_S
        res = self._pipe({"raw": samples, "sampling_rate": TARGET_SAMPLE_RATE}, **call)
        return (res["text"] if isinstance(res, dict) else str(res)).strip()

    def transcribe(self, audio, sampling_rate: int | None = None, generate_kwargs: Mapping[str, Any] | None = None,
                   self_chunks: bool = False, chunk_length_s: float = 120.0, chunk_overlap_s: float = 5.0) -> str:
        samples, sr = coerce_audio(audio, sampling_rate)
        samples = resample(samples, sr)
        if self_chunks:
            return self._run(samples, generate_kwargs)
        windows = split_waveform(samples, TARGET_SAMPLE_RATE, chunk_length_s, chunk_overlap_s)
        return merge_transcripts([self._run(w, generate_kwargs) for w in windows]).strip()


_CACHE: dict[tuple, ASRTranscriber] = {}
_CACHE_LOCK = threading.Lock()


def _frozen(v):
    if isinstance(v, dict):
        return tuple(sorted((k, _frozen(x)) for k, x in v.items()))
    if isinstance(v, (list, tuple)):
        return tuple(_frozen(x) for x in v)
    return v


def get_transcriber(model_id: str, device: str = "cuda", dtype: str | None = None, revision: str | None = None,
                    pipeline_kwargs: Mapping[str, Any] | None = None) -> ASRTranscriber:
    key = (model_id, revision, device, dtype, _frozen(dict(pipeline_kwargs or {})))
    with _CACHE_LOCK:
        t = _CACHE.get(key)
        if t is None:
            t = _CACHE[key] = ASRTranscriber(model_id, device, dtype, revision, pipeline_kwargs)
        return t


__all__ = ["ASRTranscriber", "get_transcriber", "resample", "coerce_audio", "resolve_generate_kwargs",
           "TARGET_SAMPLE_RATE"]
