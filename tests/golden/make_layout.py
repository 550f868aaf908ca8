"""Writes the byte layout (sizeof, offsetof of every field) of `struct MoEArgs`
as compiled from a given moe_args.h -- used to pin the layout of this
repository's include/moe_args.h to the reference's include/moe_args.h.

    python tests/golden/make_layout.py <dir containing moe_args.h> [out.json]
"""
from __future__ import annotations

import json
import re
import subprocess
import sys
import tempfile
from pathlib import Path

CUDA_INC = "/usr/local/cuda/include"


def fields(header: Path) -> list[str]:
    body = header.read_text().split("struct MoEArgs", 1)[1].split("};", 1)[0]
    body = re.sub(r"//[^\n]*", "", body)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if decl and decl != "{":
            names.append(re.findall(r"[A-Za-z_][A-Za-z0-9_]*", decl)[-1])
    return names


def layout(include_dir: Path) -> dict:
    header = (include_dir / "moe_args.h").resolve()
    names = fields(header)
    src = ['#include <cstdio>', '#include <cstddef>', f'#include "{header}"', 'int main() {',
           '  printf("{\\"sizeof\\": %zu, \\"fields\\": [", sizeof(MoEArgs));']
    for i, n in enumerate(names):
        sep = "" if i == 0 else ","
        src.append(f'  printf("{sep}[\\"{n}\\", %zu, %zu]", offsetof(MoEArgs, {n}), sizeof(((MoEArgs*)0)->{n}));')
    src += ['  printf("]}\\n");', '  return 0;', '}']
    with tempfile.TemporaryDirectory() as td:
        c = Path(td) / "l.cpp"
        c.write_text("\n".join(src))
        exe = Path(td) / "l"
        subprocess.run(["g++", "-std=c++17", "-I", CUDA_INC, str(c), "-o", str(exe)], check=True)
        return json.loads(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)


if __name__ == "__main__":
    res = layout(Path(sys.argv[1]))
    out = Path(sys.argv[2]) if len(sys.argv) > 2 else Path(__file__).with_name("moe_args_layout.json")
    out.write_text(json.dumps(res, indent=1) + "\n")
    print(f"wrote {out}: sizeof {res['sizeof']}, {len(res['fields'])} fields")
