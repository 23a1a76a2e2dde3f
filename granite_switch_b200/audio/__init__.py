"""Audio cascade: transcribe clips and splice the transcripts into prompts as text tokens."""
from .asr import ASRTranscriber, get_transcriber, resample
from .chunking import merge_transcripts, split_waveform
from .processor import AUDIO_MARKER, EMPTY_TRANSCRIPT_TEXT, AudioPromptProcessor

__all__ = ["ASRTranscriber", "get_transcriber", "resample", "merge_transcripts", "split_waveform",
           "AudioPromptProcessor", "AUDIO_MARKER", "EMPTY_TRANSCRIPT_TEXT"]
