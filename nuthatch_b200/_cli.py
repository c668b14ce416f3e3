"""Argument and output conventions shared by the text tools (olmoe_generate,
olmoe_stream, olmoe_trace), as the reference's *_main.cc programs have them:
C atoi for counts, the prompt as the remaining arguments joined by single
spaces, NUTHATCH_NORM_TOPK=1 to renormalise the top-k weights, and decoded
text written as raw bytes."""
from __future__ import annotations

import os
import sys
from typing import Sequence


def atoi(s: str) -> int:
    """C atoi: leading whitespace, an optional sign, then decimal digits; 0
    when there are none."""
    s = s.lstrip(" \t\n\v\f\r")
    sign, i = 1, 0
    if s[:1] in ("+", "-"):
        sign, i = (-1 if s[0] == "-" else 1), 1
    j = i
    while j < len(s) and "0" <= s[j] <= "9":
        j += 1
    return sign * int(s[i:j]) if j > i else 0


def prompt_text(argv: Sequence[str], first: int) -> str:
    return " ".join(argv[first:])


def norm_topk_from_env() -> bool:
    return os.environ.get("NUTHATCH_NORM_TOPK", "")[:1] == "1"


def emit(line: str | bytes = "") -> None:
    """One output line; bytes go out unchanged (decoded text need not be
    UTF-8)."""
    data = line if isinstance(line, bytes) else line.encode()
    sys.stdout.flush()
    buf = getattr(sys.stdout, "buffer", None)
    if buf is not None:
        buf.write(data + b"\n")
        buf.flush()
    else:
        sys.stdout.write(data.decode("utf-8", errors="replace") + "\n")
