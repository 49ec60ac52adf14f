"""CPU checks of the native libffm reader (mfm_libffm_read) against fixtures
made by the reference's own load_libffm (python/modern_fm/libffm.py:31-83;
tests/golden/make_golden.py), canonicalised with the oracle's `_prep_csr`
restatement: structure, labels and field ids exact, values bitwise (strtod
and Python's float() both round correctly), error messages verbatim."""

import numpy as np
import pytest

import golden_io
from modern_fm_b200.libffm import read_libffm_raw
from oracle import oracle as O

CASES = golden_io.load("libffm.npz")


def _write(tmp_path, case):
    p = tmp_path / (case.name + ".ffm")
    p.write_bytes(case.a["text"].tobytes())
    return p


@pytest.mark.parametrize("n_threads", [1, 4])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_reader_matches_reference_golden(tmp_path, case, n_threads):
    p = _write(tmp_path, case)
    if case["error"] is not None:
        with pytest.raises(ValueError) as ei:
            read_libffm_raw(p, n_threads)
        assert str(ei.value) == case["error"].replace("{path}", str(p))
        return
    ip, ix, dv, y, f, nf = read_libffm_raw(p, n_threads)
    a, b, c = O.prep_csr(ip, ix, dv, nf)
    assert nf == case["n_features"]
    assert np.array_equal(a, case.a["indptr"]) and np.array_equal(b, case.a["indices"])
    assert np.array_equal(c.view(np.int64), case.a["data"].view(np.int64))
    assert np.array_equal(y, case.a["y"]) and np.array_equal(f, case.a["field_ids"])


def _big_text(rng, n_rows, m):
    fields = rng.integers(0, 9, size=m)
    nl = ["\n", "\r\n", "\r"]
    out = []
    for i in range(n_rows):
        js = rng.integers(0, m, size=int(rng.integers(0, 20)))
        toks = [str(int(rng.integers(0, 2)))] + [f"{fields[j]}:{j}:{rng.normal()!r}" for j in js]
        out.append(" ".join(toks) + nl[i % 3] + ("\n" if i % 97 == 0 else ""))
    return "".join(out), fields


def test_chunked_parse_equals_one_thread(tmp_path):
    """A multi-megabyte file read by 8 threads (several chunks, chunk edges
    inside \\r\\n pairs avoided, blank lines, mixed newlines) equals the
    one-thread read exactly."""
    rng = np.random.default_rng(0)
    text, _ = _big_text(rng, 120_000, 5000)
    assert len(text) > 4 << 20
    p = tmp_path / "big.ffm"
    p.write_bytes(text.encode())
    one = read_libffm_raw(p, 1)
    many = read_libffm_raw(p, 8)
    for a, b in zip(one[:5], many[:5]):
        assert a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))
    assert one[5] == many[5]
    assert len(one[3]) == 120_000


@pytest.mark.parametrize("kind", ["token", "conflict"])
def test_chunked_errors_report_the_first_in_file_order(tmp_path, kind):
    rng = np.random.default_rng(1)
    text, fields = _big_text(rng, 100_000, 4000)
    lines = text.replace("\r\n", "\n").replace("\r", "\n").split("\n")
    # line numbers as the reference counts them (universal newlines)
    target = len(lines) * 3 // 4
    while not lines[target].strip():
        target += 1
    j = 17
    bad = "oops" if kind == "token" else f"{int(fields[j]) + 1}:{j}:1.0"
    lines[target] = lines[target] + " " + bad
    lines[target + 500] = lines[target + 500] + " also:bad"  # a later error never wins
    p = tmp_path / "err.ffm"
    p.write_bytes("\n".join(lines).encode())
    msgs = []
    for nt in (1, 8):
        with pytest.raises(ValueError) as ei:
            read_libffm_raw(p, nt)
        msgs.append(str(ei.value))
    assert msgs[0] == msgs[1]
    assert msgs[0].startswith(f"{p}:{target + 1}: ")
    if kind == "token":
        assert msgs[0].endswith("bad token 'oops'; expected field:feature:value")
    else:
        assert f"feature {j} maps to fields" in msgs[0]


def test_missing_file_is_value_error(tmp_path):
    with pytest.raises(ValueError, match="cannot open"):
        read_libffm_raw(tmp_path / "nope.ffm")


def test_values_round_like_python_float(tmp_path):
    """Every value equals Python's float() of its literal bitwise (the
    reference's reader calls float(), libffm.py:59): round-trip reprs across
    magnitudes, %g / %e forms of 1-20 digits, long digit strings with large
    exponents (correct rounding beyond the exact fast path), underscores,
    subnormals and overflow."""
    rng = np.random.default_rng(5)
    vals = []
    for _ in range(8000):
        x = float(rng.normal() * 10.0 ** rng.integers(-30, 30))
        vals += [repr(x), "%.*g" % (int(rng.integers(1, 18)), x),
                 "%.*e" % (int(rng.integers(0, 20)), x)]
    for _ in range(3000):
        vals.append(str(int(rng.integers(-10**18, 10**18))))
        vals.append("0." + "".join(map(str, rng.integers(0, 10, size=int(rng.integers(1, 25))))))
        vals.append("".join(map(str, rng.integers(0, 10, size=int(rng.integers(1, 25)))))
                    + "e" + str(int(rng.integers(-330, 310))))
    vals += ["1_000.5", "1_0e1_0", ".5", "5.", "-0", "+0.0", "1e-400", "4.9406564584124654e-324",
             "2.2250738585072011e-308", "9007199254740993", "0.1", "1e22", "1e23",
             "123456789012345e-22", "1234567890123456e-22", "-INF", "Infinity", "1.7976931348623159e308"]
    p = tmp_path / "v.ffm"
    p.write_text("".join("1 " + " ".join(f"0:{i + k}:{v}" for k, v in enumerate(vals[i:i + 10]))
                         + "\n" for i in range(0, len(vals), 10)))
    _, _, dv, _, _, _ = read_libffm_raw(p, 4)
    want = np.array([float(v) for v in vals])
    assert np.array_equal(dv.view(np.int64), want.view(np.int64))
