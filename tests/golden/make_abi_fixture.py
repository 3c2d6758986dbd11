"""Measure sizeof/offsetof of every ABI struct from a C header and write them
as JSON. Run in the build container against the reference headers:

    python tests/golden/make_abi_fixture.py /path/to/reference/include > tests/golden/abi_offsets.json

tests/test_abi.py runs the same probe against include/turbo/turbo_abi.h and
compares both, and the ctypes mirror, with this fixture.
"""
import json
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from turboembed_b200 import abi  # noqa: E402


def probe(include_dir, header):
    lines = ["#include <stdio.h>", "#include <stddef.h>", f"#include <{header}>", "int main(void) {"]
    for name, cls in abi.STRUCTS.items():
        lines.append(f'printf("{name} __size__ %zu\\n", sizeof({name}));')
        for f, *_ in cls._fields_:
            lines.append(f'printf("{name} {f} %zu\\n", offsetof({name}, {f}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src, exe = Path(d) / "p.c", Path(d) / "p"
        src.write_text("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", "-I", str(include_dir), str(src), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    res = {}
    for line in out.splitlines():
        s, f, v = line.split()
        res.setdefault(s, {})[f] = int(v)
    return res


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_abi_fixture.py <reference include directory>  (holding turbo/turbo.h)")
    inc = Path(sys.argv[1])
    print(json.dumps(probe(inc, "turbo/turbo_backend.h"), indent=1, sort_keys=True))
