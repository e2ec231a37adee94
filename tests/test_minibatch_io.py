"""The reference's raw-binary COO files (dst_local.bin / src_local.bin,
src/swtcf_spmm_main.cu:17-31, 128-142): round trip and the same rejections."""
import numpy as np
import pytest

from tcc_b200 import minibatch


def test_coo_bin_round_trip(tmp_path):
    rng = np.random.default_rng(4)
    dst = rng.integers(0, 500, 3000).astype(np.uint32)
    src = rng.integers(0, 700, 3000).astype(np.uint32)
    d, s = str(tmp_path / "dst_local.bin"), str(tmp_path / "src_local.bin")
    minibatch.write_coo_bin(d, s, dst, src)
    assert (tmp_path / "dst_local.bin").stat().st_size == 4 * 3000
    rd, rs, rows, cols = minibatch.read_coo_bin(d, s)
    assert np.array_equal(rd, dst) and np.array_equal(rs, src)
    assert rows == int(dst.max()) + 1 and cols == int(src.max()) + 1


def test_coo_bin_rejects_bad_files(tmp_path):
    d, s = tmp_path / "d.bin", tmp_path / "s.bin"
    d.write_bytes(b"\x01\x00\x00\x00\x02")  # not a multiple of 4 bytes
    s.write_bytes(b"\x01\x00\x00\x00")
    with pytest.raises(ValueError, match="invalid file size"):
        minibatch.read_coo_bin(str(d), str(s))
    d.write_bytes(b"\x01\x00\x00\x00" * 2)
    with pytest.raises(ValueError, match="invalid COO"):
        minibatch.read_coo_bin(str(d), str(s))
    d.write_bytes(b"")
    s.write_bytes(b"")
    with pytest.raises(ValueError, match="invalid COO"):
        minibatch.read_coo_bin(str(d), str(s))
