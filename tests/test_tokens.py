"""CPU test of the drop-in's token input (main.cpp:14-58, Detokenizer.cpp:41-80):
uint32 token files -> padded batch, pad id from vocab.txt.  Runs the compiled
C++ driver; no GPU work."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPP = os.path.join(ROOT, "dirktensor_b200", "cpp")


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    subprocess.run(["make", "-s", "-C", CPP], check=True)
    out = str(tmp_path_factory.mktemp("tok") / "test_dropin")
    subprocess.run(["g++", "-std=c++20", "-O2", f"-I{CPP}", f"-I{CPP}/compat", f"-I{ROOT}/include", "-o", out,
                    os.path.join(ROOT, "tests", "cpp", "test_dropin.cpp"), f"-L{CPP}", "-l:libdirktensor_dropin.so",
                    f"-Wl,-rpath,{CPP}", f"-L{ROOT}/dirktensor_b200", "-l:libdirktensor_b200.so",
                    f"-Wl,-rpath,{ROOT}/dirktensor_b200"], check=True)
    return out


def test_token_files_to_padded_batch(driver, tmp_path):
    rng = np.random.default_rng(5)
    seqs = [rng.integers(0, 100352, n).astype("<u4") for n in (7, 1, 12)]
    files = []
    for i, s in enumerate(seqs):
        p = tmp_path / f"s{i}.tokens.bin"
        s.tofile(p)
        files.append(str(p))
    # a trailing partial id is ignored, as the reference's read loop ignores it
    with open(files[0], "ab") as f:
        f.write(b"\x01\x02")
    vocab = tmp_path / "vocab.txt"
    vocab.write_text("0\t!\n1\t\"\n100277\t<|pad|>\n100278\t<|endoftext|>\n")
    r = subprocess.run([driver, "tokens", str(tmp_path), str(vocab)] + files, check=True, capture_output=True,
                       text=True)
    rows, cols, pad = (int(x) for x in r.stdout.split())
    assert (rows, cols, pad) == (3, 12, 100277)
    got = np.fromfile(tmp_path / "batch.u32", "<u4").reshape(rows, cols)
    for i, s in enumerate(seqs):
        assert np.array_equal(got[i, :len(s)], s)
        assert np.all(got[i, len(s):] == pad)


def test_missing_token_file_raises(driver, tmp_path):
    vocab = tmp_path / "vocab.txt"
    vocab.write_text("5\tx\n")
    r = subprocess.run([driver, "tokens", str(tmp_path), str(vocab), str(tmp_path / "nope.bin")],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "Cannot open file" in r.stderr
