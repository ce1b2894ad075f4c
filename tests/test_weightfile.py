"""The weight-file loader's index and checks (host only, no GPU): files
written the way weightfile/binaryfile.go writes them (weightfile_format.py)
are indexed with every parameter's storage, precision and shape, and damaged
files fail with the reference reader's errors (binaryfile.go:157-398,
lowprecision/rows.go:172-203)."""
import numpy as np
import pytest

from gotransformers_b200 import _lib
from gotransformers_b200.moe import WeightFile
from oracle import oracle as O
from weightfile_format import bf16_bits, compressed_record, write


def _layer(precision, rows, width, seed):
    rng = np.random.default_rng(seed)
    return O.quantize_rows(precision, rng.standard_normal((rows, width)) / np.sqrt(width))


def _model_params(seed=0):
    params = []
    rng = np.random.default_rng(seed)
    params.append(("router.weights", ("f64", rng.standard_normal(8 * 32))))
    params.append(("router.biases", ("f32", rng.standard_normal(8))))
    for i, prec in enumerate((O.FLOAT64, O.FLOAT32, O.INT8, O.FP4)):
        L = _layer(prec, 24, 33, seed + i)
        params.append((f"expert{i}.gate.weights", compressed_record(prec, L.rows, L.width, L.values, L.scales)))
        params.append((f"expert{i}.gate.biases", ("bf16", rng.standard_normal(24))))
    return params


def test_index_matches_what_was_written(tmp_path):
    path = tmp_path / "model.bin"
    write(str(path), _model_params())
    wf = WeightFile(str(path))
    assert wf.params["router.weights"] == (1, -1, 0, 0, 256)
    assert wf.params["router.biases"] == (2, -1, 0, 0, 8)
    for i, prec in enumerate((O.FLOAT64, O.FLOAT32, O.INT8, O.FP4)):
        assert wf.params[f"expert{i}.gate.weights"] == (4, prec, 24, 33, 24 * 33)
        assert wf.params[f"expert{i}.gate.biases"] == (3, -1, 0, 0, 24)
    wf.close()


def test_version_one_is_float64_only(tmp_path):
    path = tmp_path / "v1.bin"
    write(str(path), [("a", ("f64", np.arange(5.0))), ("b", ("f64", np.zeros(0)))], version=1)
    wf = WeightFile(str(path))
    assert wf.params == {"a": (1, -1, 0, 0, 5), "b": (1, -1, 0, 0, 0)}
    wf.close()


def test_bfloat16_rounding_matches_the_reference_rule():
    # ties to even at bfloat16 spacing (precision.go:58-71)
    assert bf16_bits(1.0) == 0x3F80
    assert bf16_bits(1.0 + 2.0 ** -8) == 0x3F80  # halfway, even stays
    assert bf16_bits(1.0 + 3 * 2.0 ** -8) == 0x3F82  # halfway, rounds up to even
    assert bf16_bits(-2.5) == 0xC020
    assert bf16_bits(float("nan")) == 0x7FC0


def _expect_error(path, needle):
    with pytest.raises(_lib.GtmoeError) as e:
        WeightFile(str(path))
    assert needle in str(e.value), str(e.value)


def test_damaged_files_fail_like_the_reference(tmp_path):
    good = tmp_path / "good.bin"
    write(str(good), _model_params())
    raw = good.read_bytes()

    bad = tmp_path / "marker.bin"
    bad.write_bytes(b"NOT-A-WEIGHTS-FILE-AT-ALL" + raw[24:])
    _expect_error(bad, "this is not a binary weights file")

    short = tmp_path / "short.bin"
    short.write_bytes(raw[:-7])
    _expect_error(short, "could not read the")

    dup = tmp_path / "dup.bin"
    write(str(dup), [("x", ("f64", np.ones(3))), ("x", ("f64", np.ones(3)))])
    _expect_error(dup, 'parameter "x" is in the file twice')

    unknown = tmp_path / "unknown.bin"
    write(str(unknown), [("x", ("f64", np.ones(3)))])
    b = bytearray(unknown.read_bytes())
    b[24 + 4 + 4 + 1] = 9  # the storage byte after the 1-byte name
    unknown.write_bytes(bytes(b))
    _expect_error(unknown, "is stored in an unknown way (9)")

    huge = tmp_path / "huge.bin"
    write(str(huge), [("x", ("f64", np.ones(3)))])
    b = bytearray(huge.read_bytes())
    b[24 + 4 + 4 + 1 + 1:24 + 4 + 4 + 1 + 1 + 8] = (1 << 40).to_bytes(8, "little")
    huge.write_bytes(bytes(b))
    _expect_error(huge, "which is more than the file can hold")

    L = _layer(O.INT8, 4, 20, 7)
    wrong = tmp_path / "wrong.bin"
    write(str(wrong), [("w", compressed_record(O.INT8, 4, 20, L.values, L.scales[:-1]))])
    _expect_error(wrong, "has the wrong amount of data")

    # the combined byte count RowsFromSnapshot checks is right, the split is
    # not: one scale fewer and four more code bytes.  The reference reader
    # accepts it and DotRow panics later; the loader refuses it up front.
    split = tmp_path / "split.bin"
    codes = np.concatenate([L.values, np.zeros(4, np.int8)])
    write(str(split), [("w", compressed_record(O.INT8, 4, 20, codes, L.scales[:-1]))])
    _expect_error(split, "holds 84 codes and 7 scales; 4 rows of width 20 need 80 and 8")
    Lf = _layer(O.FP4, 3, 33, 8)
    split4 = tmp_path / "split4.bin"
    write(str(split4), [("w", compressed_record(O.FP4, 3, 33, Lf.values[:-8], np.concatenate(
        [Lf.scales, np.ones(2, np.float32)])))])
    _expect_error(split4, "holds 43 codes and 11 scales; 3 rows of width 33 need 51 and 9")

    wide = tmp_path / "wide.bin"
    write(str(wide), [("w", compressed_record(O.INT8, 4, 0, np.zeros(0, np.int8), np.zeros(0, np.float32)))])
    _expect_error(wide, "which does not fit in the file")


def test_missing_file_and_missing_parameter(tmp_path):
    with pytest.raises(_lib.GtmoeError):
        WeightFile(str(tmp_path / "absent.bin"))
