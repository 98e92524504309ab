"""The committed ncu summaries (profiles/) are text that bench.py and readers
rely on: every ncu command in them leaves the GPU clocks alone
(--clock-control none) and runs committed files only, and the traffic lines
bench.py reads parse as numbers."""
import os
import re

import pytest

PROFILES = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "profiles")
FILES = sorted(f for f in os.listdir(PROFILES) if f.endswith((".md", ".txt")))


def test_there_are_summaries():
    assert any(f.startswith("step_config2") for f in FILES)


@pytest.mark.parametrize("name", FILES)
def test_summary_commands_follow_the_rules(name):
    text = open(os.path.join(PROFILES, name)).read()
    assert "_work" not in text
    commands = re.findall(r"^\s+ncu .*?(?=\n\s*\n|\Z)", text, flags=re.M | re.S)
    assert commands, "a summary names the command that made it"
    for cmd in commands:
        assert "--clock-control none" in cmd, cmd
        assert re.search(r"\bpython bench\.py\b", cmd), cmd
        # Anything beyond the one-pass launch list (more metrics, sections,
        # sets) replays each captured launch several times: such captures
        # name one kernel and a few launches.
        m = re.search(r"--metrics\s+(\S+)", cmd)
        heavy = ("--set" in cmd or "--section" in cmd or (m is not None and m.group(1) != "gpu__time_duration.sum"))
        if heavy:
            assert re.search(r"(^|\s)-k\s", cmd) and re.search(r"(^|\s)-c\s+[1-3]\b", cmd), \
                f"a multi-pass capture must select one kernel (-k) and 1-3 launches (-c): {cmd}"
    for ln in text.splitlines():
        if ln.startswith("bench-traffic:"):
            parts = ln.split()
            assert len(parts) == 3 and float(parts[2]) > 0, ln
