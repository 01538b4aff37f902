"""Format-preserving writes to a TOML config file: `set_value` changes one key and leaves every
other line (comments, blank lines, order, the key's own trailing comment) as it was.  The value
is checked against the schema first, so a file that loaded before still loads after.
Reference: crates/config/src/write.rs.
"""
from __future__ import annotations

import json
import os
import re

from .schema import Config

_HEADER = re.compile(r"^\s*\[([A-Za-z0-9_.-]+)\]\s*(#.*)?$")


def _toml_value(raw, cur) -> str:
    """TOML literal of `raw` for a field whose current value is `cur` (bool / int / float / list /
    str); size and duration strings ("8GiB", "500ms") stay strings."""
    if isinstance(cur, bool):
        return "true" if str(raw).strip().lower() in ("1", "true", "yes", "on") else "false"
    if isinstance(cur, list):
        items = raw if isinstance(raw, (list, tuple)) else [x for x in str(raw).split(",") if x]
        return "[" + ", ".join(json.dumps(str(x)) for x in items) + "]"
    if isinstance(cur, (int, float)):
        s = str(raw).strip()
        try:
            float(s)
            return s
        except ValueError:
            return json.dumps(s)  # "8GiB", "2s": parsed by the schema's unit types
    return json.dumps(str(raw))  # a basic string with JSON-compatible escapes


def _split_comment(line: str) -> tuple[str, str]:
    """(code, comment) of a TOML line; a '#' inside a basic string is not a comment."""
    in_str, esc = False, False
    for i, ch in enumerate(line):
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
        elif ch == '"':
            in_str = True
        elif ch == "#":
            return line[:i], line[i:]
    return line, ""


def set_value(path: str, dotted: str, raw) -> str:
    """Sets `section.key` to `raw` in the file at `path` (created when missing); returns the new
    text.  Raises KeyError for an unknown key and ValueError for a value that does not parse."""
    section, _, key = dotted.rpartition(".")
    probe = Config()
    probe.set(dotted, raw, "write")       # unknown key / unparsable value -> ValueError
    cur = getattr(getattr(Config(), section), key)
    value = _toml_value(raw, cur)
    text = open(path).read() if os.path.exists(path) else ""
    lines = text.splitlines(keepends=True)
    cur_sec, sec_line, last_in_sec = None, None, None
    for i, line in enumerate(lines):
        m = _HEADER.match(line)
        if m:
            cur_sec = m.group(1)
            if cur_sec == section:
                sec_line, last_in_sec = i, i
            continue
        if cur_sec != section:
            continue
        code, comment = _split_comment(line.rstrip("\n"))
        if code.strip():
            last_in_sec = i
        k, eq, _ = code.partition("=")
        if eq and k.strip() == key:
            indent = code[:len(code) - len(code.lstrip())]
            gap = code[len(code.rstrip()):] if comment else ""
            nl = "\n" if line.endswith("\n") else ""
            lines[i] = f"{indent}{key} = {value}{gap or (' ' if comment else '')}{comment}{nl}"
            return _commit(path, "".join(lines))
    if sec_line is None:
        sep = "" if not text or text.endswith("\n\n") else ("\n" if text.endswith("\n") else "\n\n")
        return _commit(path, f"{text}{sep}[{section}]\n{key} = {value}\n")
    if not lines[last_in_sec].endswith("\n"):
        lines[last_in_sec] += "\n"
    lines.insert(last_in_sec + 1, f"{key} = {value}\n")
    return _commit(path, "".join(lines))


def _commit(path: str, text: str) -> str:
    from .schema import load_config
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        f.write(text)
    load_config(tmp, env={})  # the written file must load
    os.replace(tmp, path)
    return text
