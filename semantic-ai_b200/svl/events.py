"""STT events for many streams: the word / timestamp / voice-activity logic of the reference's
Recognizer and TurnDetector (stt/mod.rs:263-352, :544-612) on the host, over the tokens and
extra-head probabilities of the device token loop (svl_stt_run_frames_ex).

The language-model loop (one CUDA graph per step for all streams) runs on the GPU; what is left
per stream and frame is a handful of comparisons, so it stays on the host. The tokenizer
(sentencepiece in the reference) is the caller's: an object with decode(tokens) -> str and
encode(word) -> list of token ids.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

END_OF_PADDING = 0  # stt/mod.rs:170
PADDING = 3
FRAME_RATE = 12.5   # frames per second (80 ms)


@dataclass
class Word:
    """SttEvent::Word: a word starting `start` seconds into the stream."""
    text: str
    start: float


@dataclass
class WordEnd:
    """SttEvent::WordEnd: the end of the last word, in seconds."""
    end: float


@dataclass
class VoiceActivity:
    """SttEvent::VoiceActivity: per frame, the probability of a pause for each horizon."""
    time: float
    pause_probabilities: list


def _round_ms(x: float) -> float:
    return round(x * 1000.0) / 1000.0


@dataclass
class Recognizer:
    """The language-model side of one stream (stt/mod.rs:419-428, :544-612), minus the model:
    it turns the stream's greedy text tokens and voice-activity probabilities into events.
    time_offset starts at the silence prefix plus the model's audio delay (stt/mod.rs:245)."""
    tokenizer: object
    time_offset: float = 0.0
    steps: int = 0
    word_tokens: list = field(default_factory=list)
    word_start: float = 0.0
    unended_word: bool = False

    def text_time(self, index: int) -> float:
        """Audio time of the text predicted at step `index` (stt/mod.rs:545-549)."""
        return _round_ms(max(index / FRAME_RATE - self.time_offset, 0.0))

    def step(self, token: int, extra=(), events: list | None = None) -> list:
        """One frame's prediction (Recognizer::step after LanguageModel::step)."""
        events = [] if events is None else events
        index = self.steps
        self.steps += 1
        if len(extra):
            events.append(VoiceActivity(self.text_time(index), [float(p) for p in extra]))
        # Words are separated by end-of-padding tokens and followed by padding.
        if token == END_OF_PADDING or token == PADDING:
            if self.word_tokens:
                self.emit_words(events)
        elif token > PADDING:
            self.word_tokens.append(int(token))
        if token == END_OF_PADDING:
            if self.unended_word:
                self.unended_word = False
                events.append(WordEnd(self.text_time(index)))
            self.word_start = self.text_time(index + 1)
        return events

    def emit_words(self, events: list) -> None:
        """The pending word tokens as words; words spoken quickly share a segment and each gets
        as many frames as it has tokens (stt/mod.rs:595-611)."""
        text = self.tokenizer.decode(self.word_tokens)
        self.word_tokens = []
        start = self.word_start
        for word in text.split():
            events.append(Word(word, start))
            n = len(self.tokenizer.encode(word)) or 1
            start = _round_ms(start + n / FRAME_RATE)
        self.unended_word = True

    def finish(self, end: float) -> list:
        """The tail of SttStream::flush (stt/mod.rs:470-481) once the delay's silence has gone
        through the model: the pending words, then the end of the last one at `end` (the audio
        time when the flush began), at least its start."""
        events = []
        if self.word_tokens:
            self.emit_words(events)
        if self.unended_word:
            self.unended_word = False
            events.append(WordEnd(max(end, self.word_start)))
        return events


class TurnDetector:
    """The end of a speaker's turn from a stream's voice activity (stt/mod.rs:276-352): after
    some words, the pause probability of the 2-second head above `threshold` for `frames`
    consecutive frames."""

    HEAD = 2

    def __init__(self, threshold: float = 0.5, frames: int = 1):
        self.threshold = threshold
        self.frames = max(1, frames)
        self.above = 0
        self.in_turn = False

    def update(self, event) -> bool:
        """Feeds an event; True when it ends the current turn."""
        if isinstance(event, Word):
            self.in_turn = True
            return False
        if isinstance(event, WordEnd):
            return False
        p = event.pause_probabilities
        pause = len(p) > self.HEAD and p[self.HEAD] > self.threshold
        self.above = self.above + 1 if pause else 0
        if self.in_turn and self.above >= self.frames:
            self.in_turn = False
            return True
        return False


@dataclass
class TranscriptWord:
    text: str
    start: float
    end: float


@dataclass
class Transcript:
    """Transcript::from_events (stt/mod.rs:364-397)."""
    text: str
    words: list

    @staticmethod
    def from_events(events) -> "Transcript":
        words: list[TranscriptWord] = []
        for e in events:
            if isinstance(e, Word):
                # Words sharing a segment end where the next one starts.
                if words and words[-1].end < e.start:
                    words[-1].end = e.start
                words.append(TranscriptWord(e.text, e.start, e.start))
            elif isinstance(e, WordEnd):
                if words:
                    words[-1].end = e.end
        return Transcript(" ".join(w.text for w in words), words)


class BatchedRecognizer:
    """Recognizers for streams 0..B-1 of a state, stepped together: each feed() runs the
    frames through the device token loop (one CUDA graph per step for all streams) and turns
    every stream's tokens and voice activity into its events."""

    def __init__(self, model, state, tokenizer, streams: int, time_offset: float = 0.0):
        self.model, self.state, self.streams = model, state, streams
        self.recognizers = [Recognizer(tokenizer, time_offset=time_offset) for _ in range(streams)]

    def feed(self, audio_codes: np.ndarray) -> list:
        """audio_codes [frames, B, n_q] -> per stream, the list of its events."""
        toks, extra = self.model.run_frames(audio_codes, self.state, extra=True)
        out = [[] for _ in range(self.streams)]
        for f in range(toks.shape[0]):
            for b in range(self.streams):
                self.recognizers[b].step(int(toks[f, b]), extra[f, b], out[b])
        return out
