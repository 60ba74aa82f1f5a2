"""The host side of batched STT events (svl/events.py), on CPU: the reference's TurnDetector
cases (stt/mod.rs:614-664), the Recognizer's word / timestamp / voice-activity rules
(stt/mod.rs:544-612) on synthetic token streams, and Transcript::from_events."""
from svl.events import (END_OF_PADDING, PADDING, Recognizer, Transcript, TurnDetector,
                        VoiceActivity, Word, WordEnd)


def activity(pause):
    return VoiceActivity(0.0, [0.0, 0.0, pause, 0.0])


def word():
    return Word("word", 0.0)


def ends(detector, events):
    return [detector.update(e) for e in events]


def test_turns_end_after_words_only():
    d = TurnDetector()
    # Pauses before any word are not ends of turns.
    assert ends(d, [activity(0.9), activity(0.9)]) == [False, False]
    assert ends(d, [word(), activity(0.2), activity(0.9), activity(0.9)]) == [False, False, True, False]


def test_turns_end_after_consecutive_frames():
    d = TurnDetector(threshold=0.6, frames=3)
    events = [word(), activity(0.7), activity(0.7), activity(0.5),  # a hesitation: starts over
              activity(0.7), activity(0.7), activity(0.7)]
    assert ends(d, events) == [False, False, False, False, False, False, True]


class Tok:
    """Token t > PADDING decodes to 'w<t>', one token per word; 100 + i decodes to a two-word
    text 'a<i> b<i>' (words spoken quickly share a segment)."""

    def decode(self, toks):
        out = []
        for t in toks:
            out += [f"a{t - 100}", f"b{t - 100}"] if t >= 100 else [f"w{t}"]
        return " ".join(out)

    def encode(self, word):
        return [0]


def test_recognizer_words_and_times():
    r = Recognizer(Tok(), time_offset=0.5)
    ev = []
    # step: 0 1 2 3 4 5 6 7 8 9
    for t in [PADDING, PADDING, END_OF_PADDING, 7, 8, PADDING, END_OF_PADDING, 9, PADDING, END_OF_PADDING]:
        r.step(t, (), ev)
    # Word start: text_time(index + 1) after the end of padding at step 2 = 3 / 12.5 - 0.5 = 0.0
    # (clamped); tokens 7, 8 form one segment ("w7 w8"), emitted at the padding of step 5.
    assert ev[0] == Word("w7", 0.0)
    assert ev[1] == Word("w8", 0.08)  # one token: one frame later
    # The end of padding at step 6 ends the word: text_time(6) = 0.48 - 0.5 -> 0.0 clamped,
    # then the next word starts at text_time(7) = 0.06.
    assert ev[2] == WordEnd(0.0)
    assert ev[3] == Word("w9", 0.06)
    assert ev[4] == WordEnd(round(9 / 12.5 - 0.5, 3))
    assert len(ev) == 5


def test_recognizer_shared_segment_and_voice_activity():
    r = Recognizer(Tok())
    ev = r.step(END_OF_PADDING, [0.1, 0.2, 0.3])
    assert ev == [VoiceActivity(0.0, [0.1, 0.2, 0.3])]
    r.step(103, [0.1, 0.2, 0.3])
    ev = r.step(PADDING, [])
    assert ev == [Word("a3", 0.08), Word("b3", 0.16)]
    tail = r.finish(end=0.1)
    assert tail == [WordEnd(0.1)]  # max(end of the audio, the segment start 0.08)


def test_transcript_from_events():
    t = Transcript.from_events([Word("hello", 0.1), Word("world", 0.5), WordEnd(0.9), activity(0.2)])
    assert t.text == "hello world"
    assert [(w.text, w.start, w.end) for w in t.words] == [("hello", 0.1, 0.5), ("world", 0.5, 0.9)]
