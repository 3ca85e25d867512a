"""Host-side reading of the GEMM kernels' status record (no GPU): the layout the
Python reader assumes matches the one the C header documents, and a record is
turned into the message ``check_device_status`` raises."""

import re
from pathlib import Path

from stratum_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def _record(code=0x154, block=7, thread=544, parity=0, bar=0x38470, state=0x7FFFF800001FFFFE):
    d = [0] * _lib.STATUS_WORDS
    d[0], d[1], d[2], d[3], d[4] = code, block, thread, parity, bar
    d[5], d[6] = state & 0xFFFFFFFF, state >> 32
    d[7] = 90
    ns = 2_000_123_456
    d[8], d[9] = ns & 0xFFFFFFFF, ns >> 32
    d[10] = 3_926_280_218 - (1 << 32)  # the cycle count arrives as a signed 32-bit int
    for i in range(_lib.BAR_BELOW + 1 + _lib.BAR_ABOVE):
        v = (i + 1) * 0x0101010101
        d[12 + 2 * i], d[13 + 2 * i] = v & 0xFFFFFFFF, v >> 32
    return d


def test_header_and_reader_agree_on_the_record_layout():
    text = (ROOT / "include" / "stratum_nf4.h").read_text()
    assert re.search(rf"up to {_lib.STATUS_WORDS} ints", text)
    assert re.search(rf"{_lib.BAR_BELOW} below, the\s+\* barrier, {_lib.BAR_ABOVE} above", text)
    assert 12 + 2 * (_lib.BAR_BELOW + 1 + _lib.BAR_ABOVE) <= _lib.STATUS_WORDS


def test_timeout_record_is_described():
    text = _lib.describe_status_record(_record())
    assert "block 7, thread 544, SM 90, parity 0" in text
    assert "offset 0x38470" in text and "state 0x7ffff800001ffffe" in text
    assert "2.000 s by %globaltimer and 3926280218 SM cycles" in text
    words = text.split("above: ")[1].split()
    assert len(words) == _lib.BAR_BELOW + 1 + _lib.BAR_ABOVE
    assert words[0] == f"{0x0101010101:016x}"


def test_tile_record_and_clear_word():
    d = [0] * _lib.STATUS_WORDS
    d[0], d[1], d[2], d[3], d[4], d[5], d[6] = 0x202, 3, 1, 9, 2, 100, 180
    assert _lib.describe_status_record(d) == "bad tile record: block 3, tile 1: expert 9, column tile 2, tokens [100, 180)"
    assert _lib.describe_status_record([0] * _lib.STATUS_WORDS) == ""
