"""Field offsets of the PJRT v0.55 structs, used to pin include/pjrt_b200_abi.h to the upstream ABI.

`python tests/golden/abi_offsets.py --upstream <path to xla/pjrt/c/pjrt_c_api.h>` compiles a small C
program against the upstream header (the one the reference vendors at
third_party/xla/pjrt/c/pjrt_c_api.h) and writes tests/golden/pjrt_abi_offsets.json: for every struct
that include/pjrt_b200_abi.h defines, its sizeof and the offsetof of each field.
tests/test_abi_layout.py compiles the same program against include/pjrt_b200_abi.h and compares.
"""
import argparse
import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUR_HEADER = os.path.join(ROOT, "include", "pjrt_b200_abi.h")
FIXTURE = os.path.join(HERE, "pjrt_abi_offsets.json")


def struct_fields(header_path=OUR_HEADER):
    """Parse the structs defined in our header: {name: [field, ...]} in declaration order."""
    text = open(header_path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"typedef struct (\w+) \{(.*?)\} \1;", text, flags=re.S):
        name, body = m.group(1), m.group(2)
        fields = []
        body = body.replace("PJRT_B200_HEAD;", "size_t struct_size; PJRT_Extension_Base* extension_start;")
        body = re.sub(r"union\s*\{", "", body)
        body = body.replace("};", ";")
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            fn = re.match(r"PJRT_B200_FN\(([^,]+),\s*(\w+)\)", decl)
            if fn:
                fields.append(fn.group(2))
                continue
            fp = re.search(r"\(\*(\w+)\)", decl)
            if fp:
                fields.append(fp.group(1))
                continue
            ident = re.findall(r"(\w+)\s*$", decl)
            if ident:
                fields.append(ident[0])
        out[name] = fields
    return out


def c_program(include_line, fields):
    lines = ["#include <stdio.h>", "#include <stddef.h>", include_line, "int main(void) {",
             '  printf("{\\n");']
    items = []
    for s, fs in fields.items():
        parts = ['\\"sizeof\\": %zu']
        args = [f"sizeof({s})"]
        for f in fs:
            parts.append(f'\\"{f}\\": %zu')
            args.append(f"offsetof({s}, {f})")
        items.append((s, parts, args))
    for i, (s, parts, args) in enumerate(items):
        sep = "," if i + 1 < len(items) else ""
        fmt = f'  \\"{s}\\": {{' + ", ".join(parts) + "}" + sep + "\\n"
        lines.append(f'  printf("{fmt}", {", ".join(args)});')
    lines += ['  printf("}\\n");', "  return 0;", "}"]
    return "\n".join(lines) + "\n"


def measure(include_line, fields, include_dirs=()):
    with tempfile.TemporaryDirectory() as td:
        src = os.path.join(td, "abi.c")
        exe = os.path.join(td, "abi")
        open(src, "w").write(c_program(include_line, fields))
        cmd = ["gcc", "-std=c11", "-o", exe, src] + [f"-I{d}" for d in include_dirs]
        subprocess.run(cmd, check=True, capture_output=True, text=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    return json.loads(out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--upstream", required=True, help="path to upstream pjrt_c_api.h")
    a = ap.parse_args()
    fields = struct_fields()
    got = measure(f'#include "{os.path.abspath(a.upstream)}"', fields)
    with open(FIXTURE, "w") as f:
        json.dump(got, f, indent=1, sort_keys=True)
    print(f"wrote {FIXTURE}: {len(got)} structs")


if __name__ == "__main__":
    sys.exit(main())
