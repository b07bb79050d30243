"""``__graft_entry__._ensure_reference``: the reference arm's install is
restored from a checkout when missing, left alone when present, and the
checkout is only read."""

import os

import __graft_entry__ as entry


def _fake_reference(root):
    for rel, text in (("dst/__init__.py", "X = 1\n"), ("dst/model.py", "Y = 2\n"), ("train.py", "print('t')\n"),
                      ("tests/test_a.py", "A = 3\n"), ("scripts/s.sh", "echo\n"), ("docs/notes.md", "n\n")):
        path = os.path.join(root, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            f.write(text)


def _tree(root):
    out = {}
    for d, _, files in os.walk(root):
        for f in files:
            p = os.path.join(d, f)
            out[os.path.relpath(p, root)] = open(p).read()
    return out


def test_restores_missing_install(tmp_path):
    src, dest = tmp_path / "reference", tmp_path / "repo" / "baseline" / "_ref"
    _fake_reference(str(src))
    before = _tree(str(src))
    entry._ensure_reference(str(dest), str(src))
    got = _tree(str(dest))
    assert got == {k: v for k, v in before.items() if not k.startswith("docs")}
    assert _tree(str(src)) == before


def test_present_install_and_missing_source_are_left_alone(tmp_path):
    dest = tmp_path / "_ref"
    (dest / "dst").mkdir(parents=True)
    entry._ensure_reference(str(dest), str(tmp_path / "nowhere"))
    assert os.listdir(dest) == ["dst"]
    empty = tmp_path / "empty"
    entry._ensure_reference(str(empty), str(tmp_path / "nowhere"))
    assert not empty.exists()
