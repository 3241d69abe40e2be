"""Writes tests/golden/reference_layouts.json: sizeof and every field offset of
each struct that include/prometheus_reactor.h shares (by name) with the
reference's own header, internal/prometheus/native/reactor_api.h, as gcc lays
them out on x86-64.

The reference header includes only <stdint.h>, so gcc compiles it directly;
nothing of the reference is copied: this script reads the reference header,
generates a small C program that prints offsetof / sizeof, and stores the
numbers.  tests/test_abi.py compares the repository header against them, so a
layout drift from the reference fails on CPU.

Usage (needs the reference checkout; the fixture travels with the repository):
    python tests/golden/make_layouts.py /path/to/oct
"""
from __future__ import annotations

import json
import re
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
OUR_HEADER = REPO / "include" / "prometheus_reactor.h"
FIXTURE = HERE / "reference_layouts.json"

_STRUCT = re.compile(r"typedef\s+struct\s+(\w+)\s*\{(.*?)\}\s*(\w+)\s*;", re.S)
_FIELD = re.compile(r"([\w\s\*]+?)\b(\w+)\s*(\[[^\]]*\])?\s*;")


def strip_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def parse_structs(text: str) -> dict[str, list[str]]:
    """Struct typedef name -> field names in declaration order."""
    out = {}
    for m in _STRUCT.finditer(strip_comments(text)):
        fields = [f.group(2) for f in _FIELD.finditer(m.group(2))]
        out[m.group(3)] = fields
    return out


def measure(header: Path, structs: dict[str, list[str]]) -> dict:
    """Compile a program against `header` printing sizeof and offsets of `structs`."""
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{header}"', "int main(void){"]
    for name, fields in structs.items():
        lines.append(f'printf("{name} %zu\\n", sizeof({name}));')
        for f in fields:
            lines.append(f'printf("{name}.{f} %zu\\n", offsetof({name}, {f}));')
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as td:
        src, exe = Path(td) / "layout.c", Path(td) / "layout"
        src.write_text("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
        got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                     check=True).stdout.splitlines())
    return {name: {"size": int(got[name]), "fields": [[f, int(got[f"{name}.{f}"])] for f in fields]}
            for name, fields in structs.items()}


def main(reference_root: str) -> None:
    ref_header = Path(reference_root) / "internal" / "prometheus" / "native" / "reactor_api.h"
    ours = parse_structs(OUR_HEADER.read_text())
    theirs = parse_structs(ref_header.read_text())
    shared = {name: theirs[name] for name in ours if name in theirs}
    layouts = measure(ref_header, shared)
    FIXTURE.write_text(json.dumps({"source": "internal/prometheus/native/reactor_api.h (gcc, x86-64)",
                                   "structs": layouts}, indent=1, sort_keys=True) + "\n")
    print(f"{len(layouts)} structs -> {FIXTURE}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
