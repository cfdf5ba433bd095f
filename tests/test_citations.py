"""Citations of the reference's optimizer sources point at the code they name.

Every `adamw.cpp:N[-M]` / `sgd.cpp:N[-M]` citation in the product sources, the
oracle, the bench and the design notes must lie inside the reference file,
start and end inside a function, and overlap the function the surrounding text
names (`step`, `clip_grad_norm`, `zero_grad`, the constructor,
`CosineAnnealingLR`). The function extents are
listed here; when the reference tree is present they are checked against it
(first line holds the definition, last line closes it). CPU only."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

# function -> (first line, last line) in the reference files
EXTENTS = {
    "adamw.cpp": {
        "ctor": (7, 18, "AdamW::AdamW("),
        "zero_grad": (20, 26, "void AdamW::zero_grad()"),
        "clip_grad_norm": (28, 58, "float AdamW::clip_grad_norm("),
        "step": (60, 117, "void AdamW::step()"),
        "cosine_ctor": (119, 121, "CosineAnnealingLR::CosineAnnealingLR("),
        "cosine_step": (123, 143, "void CosineAnnealingLR::step()"),
    },
    "sgd.cpp": {
        "ctor": (7, 16, "SGD::SGD("),
        "zero_grad": (18, 24, "void SGD::zero_grad()"),
        "clip_grad_norm": (26, 50, "float SGD::clip_grad_norm("),
        "step": (52, 96, "void SGD::step()"),
    },
}
FILE_LINES = {"adamw.cpp": 145, "sgd.cpp": 98}

# words in the text just before a citation that name one function (most
# specific first); a citation after one of them must overlap that function
NAMES = [
    (re.compile(r"CosineAnnealingLR|cosine|Cosine|scheduler", re.I), ("cosine_ctor", "cosine_step")),
    (re.compile(r"clip_grad_norm|clip|norm cast|grad-norm|norm"), ("clip_grad_norm",)),
    (re.compile(r"zero_grad"), ("zero_grad",)),
    (re.compile(r"AdamW::AdamW|SGD::SGD|constructor|ctor"), ("ctor",)),
    (re.compile(r"AdamW::step|SGD::step|step\(\)|per-element|element loop|moments|bias"),
     ("step",)),
]

CITE = re.compile(r"\b(adamw|sgd)\.cpp:(\d+(?:\s?[-,]\s?\d+)*)")

SCANNED = (["include", "soar.cpp_b200/csrc", "soar.cpp_b200/soar_b200", "oracle", "tests"],
           ["bench.py", "__graft_entry__.py", "DESIGN.md", "INTEGRATION.md", "README.md"])


def _files():
    dirs, files = SCANNED
    out = [ROOT / f for f in files if (ROOT / f).exists()]
    for d in dirs:
        for p in sorted((ROOT / d).rglob("*")):
            if p.is_file() and p.suffix in (".h", ".hpp", ".cu", ".cuh", ".c", ".cpp", ".py",
                                            ".md", "") and "_ref" not in p.parts:
                if p.name == Path(__file__).name:
                    continue
                out.append(p)
    return out


def _ranges(spec: str):
    for part in spec.replace(" ", "").split(","):
        if "-" in part:
            a, b = part.split("-")
            yield int(a), int(b)
        else:
            yield int(part), int(part)


def _citations():
    for p in _files():
        try:
            text = p.read_text()
        except UnicodeDecodeError:
            continue
        for lineno, line in enumerate(text.splitlines(), 1):
            for m in CITE.finditer(line):
                fname = m.group(1) + ".cpp"
                before = line[:m.start()]
                yield p.relative_to(ROOT), lineno, fname, list(_ranges(m.group(2))), before


def test_citations_found():
    cites = list(_citations())
    assert len(cites) > 20, "the citation scan found too little to be meaningful"


def test_cited_lines_lie_inside_a_function():
    bad = []
    for path, lineno, fname, ranges, _ in _citations():
        ext = EXTENTS[fname]
        for a, b in ranges:
            if not (1 <= a <= b <= FILE_LINES[fname]):
                bad.append(f"{path}:{lineno}: {fname}:{a}-{b} outside the file")
            else:
                inside = lambda x: any(lo <= x <= hi for lo, hi, _ in ext.values())
                if not (inside(a) and inside(b)):
                    bad.append(f"{path}:{lineno}: {fname}:{a}-{b} starts or ends between "
                               "functions")
    assert not bad, "\n".join(bad)


def test_cited_lines_belong_to_the_named_function():
    bad = []
    for path, lineno, fname, ranges, before in _citations():
        ctx = before[-80:]
        for rx, funcs in NAMES:
            hits = list(rx.finditer(ctx))
            if not hits:
                continue
            want = [EXTENTS[fname][f] for f in funcs if f in EXTENTS[fname]]
            if not want:
                break
            if not any(lo <= b and a <= hi for a, b in ranges for lo, hi, _ in want):
                bad.append(f"{path}:{lineno}: '{hits[-1].group(0)}' cites {fname}:{ranges}, "
                           f"not inside {funcs}")
            break
    assert not bad, "\n".join(bad)


def test_extents_match_the_reference_sources():
    from oracle import oracle
    if oracle.REF_ROOT is None:
        pytest.skip("reference sources not present")
    for fname, ext in EXTENTS.items():
        lines = (oracle.REF_ROOT / "src" / "optim" / fname).read_text().splitlines()
        assert len(lines) == FILE_LINES[fname], fname
        for name, (lo, hi, sig) in ext.items():
            assert sig in lines[lo - 1], (fname, name, lines[lo - 1])
            assert lines[hi - 1].rstrip().endswith("}"), (fname, name, lines[hi - 1])
