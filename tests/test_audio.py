"""ASR cascade on CPU: chunking and seam merge, resampling, marker expansion, engine generate."""
import numpy as np
import pytest
import torch

from granite_switch_b200.audio import (AudioPromptProcessor, EMPTY_TRANSCRIPT_TEXT, merge_transcripts, resample,
                                       split_waveform)
from granite_switch_b200.audio.asr import ASRTranscriber, resolve_generate_kwargs
from granite_switch_b200.audio.chunking import seam_overlap


def test_split_waveform_windows():
    sr = 100
    x = np.arange(1000, dtype=np.float32)          # 10 s
    segs = split_waveform(x, sr, window_s=4.0, overlap_s=1.0)
    assert [len(s) for s in segs] == [400, 400, 400]   # the window at 6 s reaches the end
    assert [int(s[0]) for s in segs] == [0, 300, 600]
    assert segs[-1][-1] == 999
    assert len(split_waveform(x, sr, 10.0, 1.0)) == 1   # one window covers the clip
    assert len(split_waveform(x[:401], sr, 4.0, 1.0)) == 2
    assert [len(s) for s in split_waveform(np.zeros(1050, np.float32), sr, 4.0, 1.0)] == [400, 400, 400, 150]
    with pytest.raises(ValueError):
        split_waveform(x, sr, 2.0, 2.0)


def test_seam_merge():
    assert seam_overlap("the quick brown fox".split(), "Brown, fox jumps".split()) == 2
    assert merge_transcripts(["the quick brown fox", "brown fox jumps over", "over the dog."]) == \
        "the quick brown fox jumps over the dog."
    assert merge_transcripts(["hello world", "", "goodbye"]) == "hello world goodbye"
    assert merge_transcripts(["a b", "c d"]) == "a b c d"


def test_resample_rate_and_tone():
    sr = 48_000
    t = np.arange(sr) / sr
    x = np.sin(2 * np.pi * 440 * t).astype(np.float32)
    y = resample(x, sr)
    assert len(y) == 16_000 and y.dtype == np.float32
    spec = np.abs(np.fft.rfft(y))
    assert abs(int(np.argmax(spec)) - 440) <= 1      # 1 Hz bins over one second


def test_transcriber_chunks_long_clips():
    seen = []

    def backend(samples):
        seen.append(len(samples))
        # each window "says" the seconds it covers: overlapping windows repeat a word
        start = int(round(samples[0]))
        return " ".join(f"w{s}" for s in range(start, start + len(samples) // 16_000))

    sr = 16_000
    x = np.repeat(np.arange(10, dtype=np.float32), sr)   # 10 s, sample value = second index
    tr = ASRTranscriber(backend=backend)
    text = tr.transcribe((x, sr), chunk_length_s=4.0, chunk_overlap_s=1.0)
    assert text == " ".join(f"w{s}" for s in range(10))
    assert seen == [64_000, 64_000, 64_000]
    assert tr.transcribe(x, sampling_rate=sr, self_chunks=True).startswith("w0 w1")
    with pytest.raises(ValueError):
        tr.transcribe(x)                                   # no rate


def test_generate_kwargs_allow_list():
    assert resolve_generate_kwargs({"num_beams": 1}, {"language": "fr"}) == {"num_beams": 1, "language": "fr"}
    with pytest.raises(ValueError):
        resolve_generate_kwargs({}, {"max_new_tokens": 5})


class _Cfg:
    asr_enabled = True
    asr_generate_kwargs = None
    asr_self_chunks = False
    asr_chunk_length_s = 120.0
    asr_chunk_overlap_s = 5.0
    asr_max_audio_clips = 2
    adapter_token_ids = [900, 901]


VOCAB = {w: i + 10 for i, w in enumerate("hello world (no speech) ctrl".split())}
VOCAB["<|a0|>"] = 900


def _encode(text):
    return [VOCAB[w] for w in text.split()]


def test_processor_expands_markers_and_guards():
    clips = {0: "hello world", 1: "", 2: "hello <|a0|>"}
    tr = ASRTranscriber(backend=lambda s: clips[int(s[0])])
    proc = AudioPromptProcessor(_Cfg(), _encode, marker_id=5, transcriber=tr)
    a = (np.zeros(1600, np.float32), 16_000)
    b = (np.ones(1600, np.float32), 16_000)
    out = proc.expand([1, 5, 2, 5, 3], [a, b])
    assert out == [1, 10, 11, 2] + _encode(EMPTY_TRANSCRIPT_TEXT) + [3]
    with pytest.raises(ValueError, match="markers"):
        proc.expand([1, 5, 2], [a, b])
    with pytest.raises(ValueError, match="exceed"):
        proc.expand([5, 5, 5], [a, a, a])
    c = (np.full(1600, 2, np.float32), 16_000)
    with pytest.raises(ValueError, match="reserved"):
        proc.expand([5], [c])


def test_engine_generate_with_audio(tmp_path):
    """A prompt with an audio marker generates exactly like the same prompt with the transcript typed in."""
    from granite_switch_b200.composer.synthetic import compose_synthetic
    from granite_switch_b200.config import GraniteSwitchConfig
    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams

    d = str(tmp_path / "m")
    compose_synthetic(d, "tiny", num_adapters=2, rank=8, num_hidden_layers=2, seed=5)
    cfg = GraniteSwitchConfig.from_pretrained(d)
    cfg.asr_enabled = True
    marker = 999
    words = {f"t{i}": 100 + i for i in range(20)}
    proc = AudioPromptProcessor(cfg, lambda s: [words[w] for w in s.split()], marker,
                                transcriber=ASRTranscriber(backend=lambda s: "t1 t2 t3 t4"))
    llm = LLM(d, device="cpu", engine_config=EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                          num_kv_blocks=32, max_model_len=128))
    sp = SamplingParams(max_tokens=4)
    with_audio = llm.generate([[7, 8, marker, 9]], sp, audios=[[(np.zeros(800, np.float32), 8000)]],
                              audio_processor=proc)[0]
    typed = llm.generate([[7, 8, 101, 102, 103, 104, 9]], sp)[0]
    assert with_audio.prompt_ids == typed.prompt_ids
    assert with_audio.output_ids == typed.output_ids
