"""Named, replaceable sections of a results markdown file (reference experiments/results_doc.py:1-42).

A section is the text between ``<!-- BEGIN:name -->`` and ``<!-- END:name -->``;
writing it again replaces only that block, so several experiments can share one
file.  The default file is ``results/results.md`` under the current directory,
or ``$MESHTRAIN_RESULTS`` when set.
"""

from __future__ import annotations

import os
import platform
import re
from datetime import datetime
from pathlib import Path

import torch


def default_path() -> Path:
    return Path(os.environ.get("MESHTRAIN_RESULTS", "results/results.md"))


def update_section(name: str, markdown: str, path: str | Path | None = None) -> Path:
    path = Path(path) if path else default_path()
    path.parent.mkdir(parents=True, exist_ok=True)
    text = path.read_text() if path.exists() else "# meshtrain_b200 results\n"
    begin, end = f"<!-- BEGIN:{name} -->", f"<!-- END:{name} -->"
    block = f"{begin}\n{markdown.rstrip()}\n{end}"
    pattern = re.compile(re.escape(begin) + r".*?" + re.escape(end), re.S)
    text = pattern.sub(lambda _m: block, text) if pattern.search(text) else text.rstrip() + "\n\n" + block + "\n"
    path.write_text(text)
    return path


def read_section(name: str, path: str | Path | None = None) -> str | None:
    path = Path(path) if path else default_path()
    if not path.exists():
        return None
    m = re.search(rf"<!-- BEGIN:{re.escape(name)} -->\n(.*?)\n<!-- END:{re.escape(name)} -->", path.read_text(), re.S)
    return m.group(1) if m else None


def environment_line() -> str:
    gpu = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "none"
    return (f"_Generated {datetime.now():%Y-%m-%d %H:%M} on {platform.node() or 'unknown'} "
            f"({platform.system()} {platform.machine()}, torch {torch.__version__}, GPU: {gpu})._")


def md_table(headers: list[str], rows: list[list]) -> str:
    lines = ["| " + " | ".join(headers) + " |", "|" + "---|" * len(headers)]
    lines += ["| " + " | ".join(str(c) for c in r) + " |" for r in rows]
    return "\n".join(lines)
