"""Native GGUF reader (inferno_gguf_*) against gguf-py on seeded files, plus
the reference reader's error cases (src/GGUF.jl:76-165): bad magic, strings
over 1 MiB, truncation, unknown value types, tensor data past the end."""
import struct

import numpy as np
import pytest

from inferno_b200 import synth as S
from inferno_b200._lib import InfernoError
from inferno_b200.gguf_file import GgufFile
from inferno_b200.model import config_from_metadata, read_gguf, spec_from_config


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=9)
    path = tmp_path_factory.mktemp("g") / "tiny.gguf"
    S.write_gguf(path, spec, T)
    return spec, T, path


def test_tensors_match_gguf_py(tiny_gguf):
    spec, T, path = tiny_gguf
    md, T2 = read_gguf(path)
    with GgufFile(path) as g:
        assert g.version == 3
        assert len(g) == len(T2)
        infos = g.tensors()
        assert [t.name for t in infos] == list(T2)           # file order
        for i, t in enumerate(infos):
            ref = T2[t.name]
            assert t.ggml_type == ref.ggml_type
            assert t.ne == tuple(ref.ne)
            assert t.nbytes == ref.data.nbytes
            assert np.array_equal(g.tensor_bytes(i), ref.data.reshape(-1)), t.name
            assert np.array_equal(g.tensor_bytes(i), T[t.name].data.reshape(-1)), t.name
        assert g.data_offset % 32 == 0


def test_metadata_and_config_match_gguf_py(tiny_gguf):
    spec, T, path = tiny_gguf
    md, T2 = read_gguf(path)
    with GgufFile(path) as g:
        nat = g.metadata()
        for k, v in md.items():
            if isinstance(v, (list, tuple)) or k.startswith("GGUF."):   # gguf-py's header pseudo-keys
                continue
            assert k in nat, k
            if isinstance(v, float):
                assert nat[k] == pytest.approx(v, rel=1e-7), k
            else:
                assert nat[k] == v, k
        assert g.get("no.such.key", 123) == 123
        assert "general.architecture" in g and "no.such.key" not in g
        infos = {t.name: t for t in g.tensors()}
        s_nat = spec_from_config(config_from_metadata(nat, infos))
        s_py = spec_from_config(config_from_metadata(md, T2))
        assert s_nat == s_py


# ---- hand-made files for the error paths ------------------------------------
def _s(x: bytes) -> bytes:
    return struct.pack("<Q", len(x)) + x


def _file(kvs=b"", nkv=0, tinfo=b"", nt=0, data=b"", magic=b"GGUF", version=3, align=32):
    head = magic + struct.pack("<IQQ", version, nt, nkv) + kvs + tinfo
    pad = (-len(head)) % align
    return head + b"\0" * pad + data


def _kv_u32(key, v):
    return _s(key) + struct.pack("<II", 4, v)


def _tensor(name, ne, ggml_type, offset):
    return _s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne) + \
        struct.pack("<IQ", ggml_type, offset)


def _open(tmp_path, blob):
    p = tmp_path / "x.gguf"
    p.write_bytes(blob)
    return GgufFile(p)


def test_minimal_file_and_alignment(tmp_path):
    data = np.arange(64, dtype=np.float32).tobytes()
    blob = _file(kvs=_kv_u32(b"general.alignment", 64), nkv=1, tinfo=_tensor(b"w", (16, 4), 0, 0), nt=1,
                 data=data, align=64)
    with _open(tmp_path, blob) as g:
        assert g.data_offset % 64 == 0
        assert g.get("general.alignment") == 64
        t = g.tensor(0)
        assert (t.name, t.ggml_type, t.ne, t.nbytes) == ("w", 0, (16, 4), 256)
        assert np.array_equal(g.tensor_bytes(0).view(np.float32), np.arange(64, dtype=np.float32))


def test_value_types(tmp_path):
    kvs = (_s(b"a.u8") + struct.pack("<IB", 0, 200) + _s(b"a.i16") + struct.pack("<Ih", 3, -5) +
           _s(b"a.f32") + struct.pack("<If", 6, 0.25) + _s(b"a.bool") + struct.pack("<IB", 7, 1) +
           _s(b"a.str") + struct.pack("<I", 8) + _s(b"hello") +
           _s(b"a.u64") + struct.pack("<IQ", 10, 2**63 + 5) + _s(b"a.f64") +
           struct.pack("<Id", 12, 1.5) +
           _s(b"a.arr") + struct.pack("<IIQ", 9, 5, 3) + struct.pack("<3i", 1, 2, 3) +
           _s(b"a.sarr") + struct.pack("<IIQ", 9, 8, 2) + _s(b"x") + _s(b"yz"))
    with _open(tmp_path, _file(kvs=kvs, nkv=9)) as g:
        assert g.get("a.u8") == 200 and g.get("a.i16") == -5 and g.get("a.bool") == 1
        assert g.get("a.f32") == 0.25 and g.get("a.f64") == 1.5 and g.get("a.str") == "hello"
        assert g.get("a.u64") == (2**63 + 5) - 2**64          # uint64 bit for bit in an int64
        assert g.get("a.arr") == (5, 3) and g.get("a.sarr") == (8, 2)
        assert g.keys()[0] == "a.u8" and len(g.keys()) == 9


@pytest.mark.parametrize("case", ["magic", "version", "long_string", "truncated", "bad_type", "past_end", "dims"])
def test_malformed_files_are_rejected(tmp_path, case):
    if case == "magic":
        blob = _file(magic=b"GGUG")
    elif case == "version":
        blob = _file(version=1)
    elif case == "long_string":                 # src/GGUF.jl:78-81: > 1 MiB is an error
        blob = _file(kvs=_s(b"k") + struct.pack("<I", 8) + struct.pack("<Q", (1 << 20) + 1) + b"a" * ((1 << 20) + 1),
                     nkv=1)
    elif case == "truncated":
        blob = _file(kvs=_kv_u32(b"key", 1), nkv=1)[:30]   # cut inside the first key
    elif case == "bad_type":
        blob = _file(kvs=_s(b"k") + struct.pack("<II", 13, 0), nkv=1)
    elif case == "past_end":
        blob = _file(tinfo=_tensor(b"w", (256, 4), 0, 0), nt=1, data=b"\0" * 100)
    else:
        blob = _file(tinfo=_s(b"w") + struct.pack("<I", 5) + b"\0" * 60, nt=1)
    with pytest.raises(InfernoError) as ei:
        _open(tmp_path, blob)
    assert ei.value.rc == -8


def test_missing_file_and_bad_key_types(tmp_path):
    with pytest.raises(InfernoError):
        GgufFile(tmp_path / "absent.gguf")
    from inferno_b200._lib import lib
    import ctypes as C
    with _open(tmp_path, _file(kvs=_kv_u32(b"k", 7), nkv=1)) as g:
        s = C.c_char_p()
        assert lib().inferno_gguf_get_string(g.h, b"k", C.byref(s)) == -1
        v = C.c_int64()
        assert lib().inferno_gguf_get_int(g.h, b"nope", C.byref(v)) == -7


def test_corrupted_headers_never_read_out_of_bounds(tiny_gguf, tmp_path):
    """Random byte flips and truncations of the header / metadata / tensor
    table: the reader either parses the file or reports it malformed."""
    _, _, path = tiny_gguf
    blob = bytearray(path.read_bytes())
    with GgufFile(path) as g:
        head = g.data_offset
    rng = np.random.default_rng(77)
    outcomes = {"ok": 0, "error": 0}
    for trial in range(300):
        b = bytearray(blob[: head + 4096]) if trial % 3 else bytearray(blob)
        for _ in range(int(rng.integers(1, 6))):
            b[int(rng.integers(0, head))] = int(rng.integers(0, 256))
        if trial % 5 == 0:
            b = b[: int(rng.integers(24, len(b)))]
        p = tmp_path / f"c{trial}.gguf"
        p.write_bytes(bytes(b))
        try:
            with GgufFile(p) as g:
                for i in range(len(g)):
                    t = g.tensor(i)
                    if t.nbytes:
                        g.tensor_bytes(i)          # must stay inside the mapping
                g.metadata()
            outcomes["ok"] += 1
        except InfernoError:
            outcomes["error"] += 1
        p.unlink()
    assert outcomes["error"] > 0 and sum(outcomes.values()) == 300


def test_plain_c_consumer(tiny_gguf, tmp_path):
    """The header compiles as C99 and a C program links against the library
    and reads the GGUF table through the C ABI (no GPU call)."""
    import shutil
    import subprocess
    from pathlib import Path
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    root = Path(__file__).resolve().parents[1]
    libdir = root / "inferno.jl_b200" / "lib"
    _, T, path = tiny_gguf
    src = tmp_path / "reader.c"
    src.write_text(r'''
#include <stdio.h>
#include "inferno_b200.h"
int main(int argc, char** argv) {
  InfernoGguf* g = 0;
  if (inferno_gguf_open(argv[1], &g)) { printf("error %s\n", inferno_last_error()); return 1; }
  const char* arch = 0;
  inferno_gguf_get_string(g, "general.architecture", &arch);
  long long n = (long long)inferno_gguf_n_tensors(g);
  unsigned long long total = 0;
  for (long long i = 0; i < n; ++i) {
    uint64_t nb = 0;
    inferno_gguf_tensor_info(g, i, 0, 0, 0, &nb, 0);
    total += nb;
  }
  printf("%s %lld %llu\n", arch, n, total);
  inferno_gguf_close(g);
  return 0;
}
''')
    exe = tmp_path / "reader"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", str(root / "include"), str(src), "-o", str(exe),
                    "-L", str(libdir), "-linferno_b200", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe), str(path)], capture_output=True, text=True, check=True).stdout.split()
    assert out[0] == "qwen35"
    assert int(out[1]) == len(T)
    assert int(out[2]) == sum(t.data.nbytes for t in T.values())


# ---- the reference's GGUF unit cases (tests/unit/test_gguf.jl:53-282), as files
def _kv(key: bytes, vtype: int, payload: bytes) -> bytes:
    return _s(key) + struct.pack("<I", vtype) + payload


def test_reference_string_cases(tmp_path):
    """read_string (:53-118): short, empty, UTF-8, 1 MiB - 1 and exactly
    1 MiB accepted; 1 MiB + 1, 100 MiB and 2^64 - 1 lengths rejected."""
    ok = [b"Hello", b"", "Hello 世界!".encode(), b"a" * 1048575, b"b" * 1048576]
    kvs = b"".join(_kv(f"s{i}".encode(), 8, _s(v)) for i, v in enumerate(ok))
    with _open(tmp_path, _file(kvs=kvs, nkv=len(ok))) as g:
        for i, v in enumerate(ok):
            assert g.get(f"s{i}") == v.decode()
    for bad_len in (1048577, 100 * 1048576, 2**64 - 1):
        blob = _file(kvs=_s(b"k") + struct.pack("<IQ", 8, bad_len) + b"x" * 64, nkv=1)
        with pytest.raises(InfernoError) as ei:
            _open(tmp_path, blob)
        assert ei.value.rc == -8


def test_reference_value_cases(tmp_path):
    """read_value (:120-272): every scalar type, strings, int32 / string /
    empty arrays; an unknown type is an error."""
    cases = [(b"u8", 0, struct.pack("<B", 42), 42), (b"i8", 1, struct.pack("<b", -42), -42),
             (b"u16", 2, struct.pack("<H", 1000), 1000), (b"i16", 3, struct.pack("<h", -1000), -1000),
             (b"u32", 4, struct.pack("<I", 100000), 100000), (b"i32", 5, struct.pack("<i", -100000), -100000),
             (b"u64", 10, struct.pack("<Q", 10000000000), 10000000000),
             (b"i64", 11, struct.pack("<q", -10000000000), -10000000000),
             (b"t", 7, b"\x01", 1), (b"f", 7, b"\x00", 0), (b"w", 8, _s(b"World"), "World")]
    kvs = b"".join(_kv(k, t, p) for k, t, p, _ in cases)
    kvs += _kv(b"f32", 6, struct.pack("<f", 3.14159)) + _kv(b"f64", 12, struct.pack("<d", 3.14159265358979))
    kvs += _kv(b"ai", 9, struct.pack("<IQ", 5, 3) + struct.pack("<3i", 1, 2, 3))
    kvs += _kv(b"as", 9, struct.pack("<IQ", 8, 2) + _s(b"Hi") + _s(b"World"))
    kvs += _kv(b"ae", 9, struct.pack("<IQ", 5, 0))
    with _open(tmp_path, _file(kvs=kvs, nkv=len(cases) + 5)) as g:
        for k, _, _, want in cases:
            assert g.get(k.decode()) == want, k
        assert abs(g.get("f32") - 3.14159) < 1e-5
        assert abs(g.get("f64") - 3.14159265358979) < 1e-14
        assert g.get_array("ai").tolist() == [1, 2, 3]
        assert g.get("as") == (8, 2)
        with pytest.raises(ValueError):
            g.get_array("as")
        assert g.get_array("ae").size == 0
    with pytest.raises(InfernoError):
        _open(tmp_path, _file(kvs=_kv(b"k", 999, b"\0" * 16), nkv=1))


def test_reference_invalid_magic(tmp_path):
    """read_gguf (:282-290): magic 0x12345678 is not a GGUF file."""
    p = tmp_path / "bad.gguf"
    p.write_bytes(struct.pack("<I", 0x12345678) + b"\0" * 60)
    with pytest.raises(InfernoError) as ei:
        GgufFile(p)
    assert ei.value.rc == -8 and "magic" in str(ei.value)
