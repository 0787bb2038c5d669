"""Generates tests/golden/reference_launchers.json: every function the
reference's host code declares inside an `extern "C"` block and therefore
links against (acediaR src/*.cpp and src/*.h; the launchers themselves are
defined in src/kernels/*.cu).  Each entry records the name and the file:line
of its declaration.

The list is parsed from the sources as text; no reference code is built or
run.  Run:  ACEDIAR_REF=<acediaR checkout> python tests/golden/make_launcher_names.py
(default checkout: /root/reference).
"""
import json
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("ACEDIAR_REF", "/root/reference")


def _strip_comments(text):
    # keep line numbers: replace comment bodies by the same count of newlines
    text = re.sub(r"/\*.*?\*/", lambda m: "\n" * m.group(0).count("\n"), text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def _blocks(text):
    """(start offset, body) of each `extern "C" { ... }` block."""
    for m in re.finditer(r'extern\s+"C"\s*\{', text):
        depth, i = 1, m.end()
        while depth and i < len(text):
            depth += {"{": 1, "}": -1}.get(text[i], 0)
            i += 1
        yield m.end(), text[m.end():i - 1]


def parse(src_dir):
    out = {}
    for fn in sorted(os.listdir(src_dir)):
        if not fn.endswith((".cpp", ".h")):
            continue
        text = _strip_comments(open(os.path.join(src_dir, fn)).read())
        for start, body in _blocks(text):
            # a declaration: <return type> name ( ... ) ;
            for m in re.finditer(r"\b([A-Za-z_]\w*)\s*\(([^;{}]*)\)\s*;", body):
                name = m.group(1)
                if name in ("if", "for", "while", "return", "sizeof"):
                    continue
                line = text.count("\n", 0, start + m.start()) + 1
                out.setdefault(name, "src/%s:%d" % (fn, line))
    return out


def main():
    names = parse(os.path.join(REF, "src"))
    doc = {"source": "extern \"C\" declarations in acediaR src/*.cpp and src/*.h (tests/golden/make_launcher_names.py)",
           "launchers": [{"name": k, "declared": v} for k, v in sorted(names.items())]}
    with open(os.path.join(HERE, "reference_launchers.json"), "w") as f:
        json.dump(doc, f, indent=1)
    print("%d names" % len(names))


if __name__ == "__main__":
    main()
