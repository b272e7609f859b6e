"""The safetensors reader (b200q8_st_*): layout and validation on the host, no GPU.

Layout as vvllm's SafeTensorsLoader reads it (src/safetensors/safetensors.cc:43-83); every
malformed header must give an error status, never a crash or an out-of-range pointer."""
import json
import struct

import numpy as np
import pytest

from tests import st_util

ERR_INVALID, ERR_IO, ERR_NOT_FOUND = -1, -7, -8


def _status(excinfo):
    return excinfo.value.status


def test_read_all_dtypes(tmp_path):
    import vvllm_b200 as v

    rng = np.random.default_rng(1)
    t = {
        "model.embed_tokens.weight": ("F32", rng.standard_normal((10, 8)).astype(np.float32)),
        "a.bf16": ("BF16", st_util.bf16_bits(rng.standard_normal((3, 5)))),
        "half": ("F16", rng.standard_normal(7).astype(np.float16)),
        "q": ("I8", rng.integers(-127, 128, (4, 6), dtype=np.int8)),
        "ids": ("I32", np.arange(5, dtype=np.int32)),
        "scalar": ("F32", np.array(3.5, np.float32)),
        "empty": ("F32", np.zeros((0, 4), np.float32)),
        'weïrd "name"\n': ("U8", np.arange(3, dtype=np.uint8)),
    }
    p = str(tmp_path / "a.safetensors")
    st_util.write(p, t, {"format": "pt"})
    with v.SafeTensors(p) as f:
        assert len(f) == len(t)
        assert sorted(f.names()) == sorted(t)
        for name, (dt, arr) in t.items():
            i = f.find(name)
            n, code, shape, _, nb = f.info(i)
            assert n == name and shape == arr.shape and nb == arr.nbytes
            assert code == {"F32": v.ST_F32, "BF16": v.ST_BF16, "F16": v.ST_F16, "I8": v.ST_I8}.get(dt, v.ST_OTHER)
            got = f.tensor(name)
            assert got.tobytes() == np.ascontiguousarray(arr).tobytes()
        with pytest.raises(v.B200Q8Error) as e:
            f.find("missing")
        assert _status(e) == ERR_NOT_FOUND
        with pytest.raises(v.B200Q8Error) as e:
            f.quantized("model.embed_tokens.weight")
        assert _status(e) == ERR_NOT_FOUND


def test_quantized_pair_views(tmp_path):
    import vvllm_b200 as v

    q = np.arange(-6, 6, dtype=np.int8).reshape(3, 4)
    s = np.array([0.5, 1.0, 2.0], np.float32)
    p = str(tmp_path / "q.safetensors")
    st_util.write(p, {"w.q8": ("I8", q), "w.q8_scales": ("F32", s), "bad.q8": ("I8", q),
                      "bad.q8_scales": ("F32", np.ones(2, np.float32))})
    with v.SafeTensors(p) as f:
        gq, gs = f.quantized("w")
        assert np.array_equal(gq, q) and np.array_equal(gs, s)
        with pytest.raises(v.B200Q8Error) as e:
            f.quantized("bad")  # scales row count differs from q's
        assert _status(e) == ERR_INVALID


def _raw(path, header_bytes, data=b"", hlen=None):
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(header_bytes) if hlen is None else hlen) + header_bytes + data)


BAD_HEADERS = [
    ("not json", b"{not json", b""),
    ("array root", b"[1,2]", b""),
    ("trailing", b'{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}} x', b"\0" * 4),
    ("no dtype", b'{"a":{"shape":[1],"data_offsets":[0,4]}}', b"\0" * 4),
    ("bad dtype", b'{"a":{"dtype":"F33","shape":[1],"data_offsets":[0,4]}}', b"\0" * 4),
    ("offsets out", b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}', b"\0" * 4),
    ("size mismatch", b'{"a":{"dtype":"F32","shape":[3],"data_offsets":[0,8]}}', b"\0" * 8),
    ("reversed", b'{"a":{"dtype":"F32","shape":[0],"data_offsets":[8,4]}}', b"\0" * 8),
    ("negative", b'{"a":{"dtype":"F32","shape":[-1],"data_offsets":[0,4]}}', b"\0" * 4),
    ("float dim", b'{"a":{"dtype":"F32","shape":[1.5],"data_offsets":[0,4]}}', b"\0" * 4),
    ("overlap", b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},'
                b'"b":{"dtype":"F32","shape":[2],"data_offsets":[4,12]}}', b"\0" * 12),
    ("duplicate", b'{"a":{"dtype":"I8","shape":[1],"data_offsets":[0,1]},'
                  b'"a":{"dtype":"I8","shape":[1],"data_offsets":[1,2]}}', b"\0" * 2),
    ("huge dims", b'{"a":{"dtype":"F32","shape":[4294967296,4294967296],"data_offsets":[0,4]}}', b"\0" * 4),
    ("meta not str", b'{"__metadata__":{"k":1}}', b""),
    ("bad escape", b'{"a\\q":{"dtype":"I8","shape":[1],"data_offsets":[0,1]}}', b"\0"),
    ("lone surrogate", b'{"a\\udc00":{"dtype":"I8","shape":[1],"data_offsets":[0,1]}}', b"\0"),
    ("deep", b"[" * 100 + b"]" * 100, b""),
    ("bad utf-8", b'{"a\xff":{"dtype":"I8","shape":[1],"data_offsets":[0,1]}}', b"\0"),
    ("overlong utf-8", b'{"\xc0\xaf":{"dtype":"I8","shape":[1],"data_offsets":[0,1]}}', b"\0"),
    ("utf-8 surrogate", b'{"\xed\xa0\x80":{"dtype":"I8","shape":[1],"data_offsets":[0,1]}}', b"\0"),
]


@pytest.mark.parametrize("name,header,data", BAD_HEADERS, ids=[b[0] for b in BAD_HEADERS])
def test_malformed_headers_rejected(tmp_path, name, header, data):
    import vvllm_b200 as v

    p = str(tmp_path / "bad.safetensors")
    _raw(p, header, data)
    with pytest.raises(v.B200Q8Error) as e:
        v.SafeTensors(p)
    assert _status(e) == ERR_INVALID, name


def test_truncated_and_missing_files(tmp_path):
    import vvllm_b200 as v

    p = str(tmp_path / "short.safetensors")
    with open(p, "wb") as fh:
        fh.write(b"\x01\x02\x03")
    with pytest.raises(v.B200Q8Error) as e:
        v.SafeTensors(p)
    assert _status(e) == ERR_INVALID
    _raw(p, b'{"a":{}}', hlen=1 << 40)  # header length past the end
    with pytest.raises(v.B200Q8Error) as e:
        v.SafeTensors(p)
    assert _status(e) == ERR_INVALID
    with pytest.raises(v.B200Q8Error) as e:
        v.SafeTensors(str(tmp_path / "nope.safetensors"))
    assert _status(e) == ERR_IO


def test_escapes_and_unicode_names(tmp_path):
    import vvllm_b200 as v

    name = "café/€/\U0001F600\t"
    hdr = json.dumps({name: {"dtype": "I8", "shape": [2], "data_offsets": [0, 2]}}, ensure_ascii=True).encode()
    p = str(tmp_path / "u.safetensors")
    _raw(p, hdr, b"\x05\x06")
    with v.SafeTensors(p) as f:
        assert f.names() == [name]
        assert f.tensor(name).tolist() == [5, 6]


def test_header_fuzz_never_crashes(tmp_path):
    """Seeded byte mutations of a valid header (flips, truncations, inserted bytes, changed
    length word): every open either succeeds with consistent metadata or returns an error status."""
    import random

    import vvllm_b200 as v

    good = str(tmp_path / "good.safetensors")
    st_util.write(good, {"a.weight": ("F32", np.arange(12, dtype=np.float32).reshape(3, 4)),
                         "b": ("I8", np.arange(5, dtype=np.int8)), "c": ("BF16", np.ones((2, 2), np.uint16))},
                  {"k": "v"})
    raw = open(good, "rb").read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    rng = random.Random(1234)
    p = str(tmp_path / "fuzz.safetensors")
    opened = failed = 0
    for _ in range(400):
        b = bytearray(raw)
        op = rng.randrange(4)
        if op == 0:  # flip bytes inside the header
            for _ in range(rng.randint(1, 4)):
                b[8 + rng.randrange(hlen)] = rng.randrange(256)
        elif op == 1:  # truncate anywhere
            b = b[:rng.randrange(len(b))]
        elif op == 2:  # insert a byte into the header, keeping the length word
            i = 8 + rng.randrange(hlen)
            b[i:i] = bytes([rng.randrange(256)])
        else:  # corrupt the length word
            b[:8] = struct.pack("<Q", rng.choice([0, 1, hlen - 1, hlen + 1, 1 << 33, rng.randrange(1 << 64)]))
        with open(p, "wb") as fh:
            fh.write(bytes(b))
        try:
            with v.SafeTensors(p) as f:
                for i in range(len(f)):
                    name, _, shape, _, nb = f.info(i)
                    assert nb >= 0 and isinstance(name, str)
            opened += 1
        except v.B200Q8Error as e:
            assert e.status in (-1, -7)
            failed += 1
    assert failed > 0 and opened + failed == 400
