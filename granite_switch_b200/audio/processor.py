"""Prompt-side audio processing: replace every ``<|audio|>`` marker by its clip's transcript ids.

An audio-enabled checkpoint adds one ``<|audio|>`` token; a prompt carries one
marker per clip, in order. Each clip is transcribed (:mod:`.asr`) and the
marker is replaced by the transcript's token ids, so the decoder, the
routing scan and the prefix cache only ever see text tokens (reference:
src/granite_switch/vllm/audio/processor.py:238-639). Rules kept from the
reference:

* the number of markers must equal the number of clips, at most
  ``asr_max_audio_clips``;
* a clip that transcribes to nothing (silence, music) becomes the text
  ``EMPTY_TRANSCRIPT_TEXT`` so the prompt keeps an audio turn;
* a transcript that tokenizes into a reserved id (the audio marker or any
  adapter control token) is refused: audio content must never steer adapter
  selection.
"""
from __future__ import annotations

from typing import Any, Callable, Mapping, Sequence

from .asr import ASRTranscriber, get_transcriber, resolve_generate_kwargs

AUDIO_MARKER = "<|audio|>"
EMPTY_TRANSCRIPT_TEXT = "(no speech)"


class AudioPromptProcessor:
    """``expand(prompt_ids, audios)`` -> prompt ids with transcripts spliced in.

    ``encode`` maps text to token ids (no special tokens added); ``marker_id`` is
    the id of ``<|audio|>``. ``transcriber`` defaults to the cached pipeline for
    the checkpoint's ASR model.
    """

    def __init__(self, config, encode: Callable[[str], list[int]], marker_id: int,
                 transcriber: ASRTranscriber | None = None):
        if not getattr(config, "asr_enabled", False):
            raise ValueError("this checkpoint was composed without audio (asr_enabled is false)")
        self.config = config
        self.encode = encode
        self.marker_id = int(marker_id)
        self._transcriber = transcriber

    @property
    def transcriber(self) -> ASRTranscriber:
        if self._transcriber is None:
            cfg = self.config
            model = cfg.asr_bundled_path or cfg.asr_model_id
            self._transcriber = get_transcriber(model, device=cfg.asr_device, dtype=cfg.asr_dtype,
                                                revision=None if cfg.asr_bundled_path else cfg.asr_model_revision,
                                                pipeline_kwargs=cfg.asr_pipeline_kwargs)
        return self._transcriber

    def reserved_ids(self) -> set[int]:
        return {self.marker_id} | {int(t) for t in (self.config.adapter_token_ids or [])}

    def transcript_ids(self, audio, request_generate_kwargs: Mapping[str, Any] | None = None) -> list[int]:
        cfg = self.config
        gk = resolve_generate_kwargs(cfg.asr_generate_kwargs, request_generate_kwargs)
        text = self.transcriber.transcribe(audio, generate_kwargs=gk or None, self_chunks=cfg.asr_self_chunks,
                                           chunk_length_s=cfg.asr_chunk_length_s,
                                           chunk_overlap_s=cfg.asr_chunk_overlap_s)
        if not text.strip():
            text = EMPTY_TRANSCRIPT_TEXT
        ids = [int(t) for t in self.encode(text)]
        if not ids:
            raise ValueError(f"the tokenizer produced no tokens for {text!r}")
        bad = sorted(set(ids) & self.reserved_ids())
        if bad:
            raise ValueError(f"transcript tokenized into reserved control token ids {bad}; refusing to splice it "
                             "into the prompt (audio content must not select adapters)")
        return ids

    def expand(self, prompt_ids: Sequence[int], audios: Sequence | None,
               request_generate_kwargs: Mapping[str, Any] | None = None) -> list[int]:
        audios = list(audios or [])
        marks = [i for i, t in enumerate(prompt_ids) if int(t) == self.marker_id]
        if len(marks) != len(audios):
            raise ValueError(f"prompt has {len(marks)} {AUDIO_MARKER} markers but {len(audios)} audio clips were given")
        if len(audios) > self.config.asr_max_audio_clips:
            raise ValueError(f"{len(audios)} audio clips exceed asr_max_audio_clips={self.config.asr_max_audio_clips}")
        out: list[int] = []
        prev = 0
        for pos, clip in zip(marks, audios):
            out.extend(int(t) for t in prompt_ids[prev:pos])
            out.extend(self.transcript_ids(clip, request_generate_kwargs))
            prev = pos + 1
        out.extend(int(t) for t in prompt_ids[prev:])
        return out


__all__ = ["AudioPromptProcessor", "AUDIO_MARKER", "EMPTY_TRANSCRIPT_TEXT"]
