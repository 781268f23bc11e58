"""Terminal presentation (colour, headings, fixed-width tables) and the interactive console.

Colour only on a TTY and never with ``NO_COLOR`` or ``TERM=dumb``
(reference terminal.py:1-151).
"""

from __future__ import annotations

import cmd
import os
import shlex
import sys

TONES = {"accent": "36", "good": "32", "warn": "33", "bad": "31", "dim": "90", "bold": "1"}
STATUS_TONES = {"ONLINE": "good", "COMPLETED": "good", "RUNNING": "warn", "BUSY": "warn", "FAILED": "bad",
                "OFFLINE": "bad", "STOPPED": "dim", "PLANNED": "dim"}
LOGO = r"""                 _     _             _         _
 _ __ ___   ___ | |__ | |_ _ __ __ _(_)_ __   | |__ ___  ___   ___
| '_ ` _ \ / _ \| '_ \| __| '__/ _` | | '_ \  | '_ \__ \/ _ \ / _ \
| | | | | |  __/| | | | |_| | | (_| | | | | | | |_) / _/ (_) | (_) |
|_| |_| |_|\___||_| |_|\__|_|  \__,_|_|_| |_| |_.__/____\___/ \___/"""


def color_enabled() -> bool:
    return sys.stdout.isatty() and "NO_COLOR" not in os.environ and os.environ.get("TERM") != "dumb"


def paint(text: str, tone: str = "accent") -> str:
    return f"\033[{TONES[tone]}m{text}\033[0m" if color_enabled() else text


def heading(title: str, detail: str = "") -> str:
    return paint(title, "bold") + (f"  {paint(detail, 'dim')}" if detail else "")


def banner() -> str:
    return paint(LOGO, "accent") + "\n" + paint("  pipeline-parallel training, B200-native", "dim")


def _clip(value, width: int) -> str:
    text = "".join(ch for ch in str(value) if ch.isprintable())
    return text if len(text) <= width else text[:max(0, width - 3)] + "..."


def table(headers: list[str], rows: list[list], widths: list[int]) -> str:
    def line(values, header=False):
        cells = []
        for v, w in zip(values, widths):
            text = _clip(v, w)
            tone = "accent" if header or text in ("CUDA", "MPS", "CPU") else STATUS_TONES.get(text)
            padded = f"{text:<{w}}"
            cells.append(paint(padded, tone) if tone else padded)
        return "  ".join(cells).rstrip()

    return "\n".join([line(headers, True), paint("  ".join("-" * w for w in widths), "dim"),
                      *(line(r) for r in rows)])


TOOLS = [
    ("CLUSTER", [("start", "start a coordinator and a worker on this machine"),
                 ("join CODE", "join another machine (CODE = TOKEN@HOST[:PORT])"),
                 ("status", "workers and their devices"),
                 ("benchmark", "measure compute and worker-to-worker links")]),
    ("TRAINING", [("plan CONFIG", "preview the placement of a config"),
                  ("inspect placement CONFIG", "stages, memory and communication in detail"),
                  ("train CONFIG", "train on the cluster"),
                  ("train CONFIG --local", "train with every stage as a local process or GPU"),
                  ("experiment NAME", "correctness / placement / capacity / device-correctness")]),
    ("MONITOR", [("jobs", "run status, loss and step time"),
                 ("dashboard", "live metrics in a local browser")]),
]


def tools_help() -> str:
    out = []
    for group, tools in TOOLS:
        out.append(paint(group, "accent"))
        out += [f"  {paint(f'{c:<34}', 'bold')}{paint(h, 'dim')}" for c, h in tools]
        out.append("")
    return "\n".join(out).rstrip()


class Console(cmd.Cmd):
    """``meshtrain console``: the CLI's commands at a prompt, sharing one coordinator/token."""

    def __init__(self, args=None, runner=None, **kw):
        super().__init__(**kw)
        self.flags: list[str] = []
        for name in ("coordinator", "token"):
            v = getattr(args, name, None) if args is not None else None
            if v:
                self.flags += [f"--{name}", v]
        self.runner = runner
        self.prompt = paint("meshtrain", "accent") + paint(" > ", "dim")
        self.intro = banner() + "\n\n" + tools_help() + "\n\n" + paint("exit to leave", "dim")

    def emptyline(self):
        return False  # never repeat the last (possibly long) command

    def default(self, line):
        if line.strip() in ("exit", "quit", "EOF"):
            return True
        try:
            argv = shlex.split(line)
        except ValueError as exc:
            print(paint(f"error: {exc}", "bad"))
            return False
        if not argv:
            return False
        if argv[0] in ("console", "start", "join"):
            print(paint(f"'{argv[0]}' is not available inside the console", "warn"))
            return False
        runner = self.runner
        if runner is None:
            from meshtrain_b200.cli import main as runner
        try:
            runner(argv + self.flags)
        except SystemExit:
            pass
        except KeyboardInterrupt:
            print(paint("cancelled", "dim"))
        except Exception as exc:  # noqa: BLE001 - a failed command must not end the console
            print(paint(f"error: {type(exc).__name__}: {exc}", "bad"))
        return False

    def do_help(self, arg):
        print(tools_help())

    def do_exit(self, arg):
        return True

    do_quit = do_exit
    do_EOF = do_exit


def run_console(args=None) -> None:
    try:
        Console(args).cmdloop()
    except KeyboardInterrupt:
        print()
