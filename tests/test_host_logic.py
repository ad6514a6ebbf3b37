"""Host-side logic of respect_b200 (no GPU): the trie / acceptance mirror against
the reference's golden vectors, and the C ABI surface of the native library."""
import ctypes
import json
import re
from pathlib import Path

import numpy as np

from respect_b200.candidates.trie import build_trie, trie_ancestry
from respect_b200.decoding.acceptance import walk

ROOT = Path(__file__).resolve().parents[1]
G = ROOT / "tests" / "golden"


def test_trie_and_walk_match_reference_golden():
    for c in json.loads((G / "trie.json").read_text()):
        t = build_trie([tuple(s) for s in c["seqs"]])
        nodes = [[n.token, -1 if n.parent is None else n.parent, n.depth] for n in t.nodes]
        assert nodes == c["nodes"], c["name"]
        assert [[k, v] for k, v in t.roots.items()] == c["roots"]
        assert [list(s) for s in t.seqs] == c["unique"]
        anc = trie_ancestry(t)
        assert [np.flatnonzero(anc[i]).tolist() for i in range(len(t.nodes))] == c["ancestry"]
        assert np.array_equal(t.parents(), np.array([n[1] for n in nodes], np.int32))
        assert np.array_equal(t.depths(), np.array([n[2] for n in nodes], np.int32))
        for w in c["walks"]:
            tg = {int(k): v for k, v in w["target"].items()}
            path, acc, rec = walk(t, w["first"], w["cap"], w["eos"], lambda a, ch: tg[ch])
            assert (path, acc, rec) == (w["path"], w["acc"], w["rec"])


def test_reference_trie_unit_cases():
    eos = 99
    t = build_trie([(1, 2, 3, eos), (1, 2, 4, eos), (1, 2, 3, eos)])
    assert [n.token for n in t.nodes] == [1, 2, 3, eos, 4, eos] and len(t.seqs) == 2
    t = build_trie([(1, 2, 3), (1, 5)])
    assert all(n.parent is None or n.parent < i for i, n in enumerate(t.nodes))
    assert np.flatnonzero(trie_ancestry(t)[3]).tolist() == [0, 3]
    t = build_trie([(1, 2, 3, eos)])
    target = {0: 2, 1: 9}
    assert walk(t, 1, 128, eos, lambda a, ch: target[ch]) == ([0, 1], [1, 2], 9)
    t = build_trie([(1, eos)])
    assert walk(t, 1, 128, eos, lambda a, ch: eos)[1] == [1, eos]
    # empty trie / unknown first token: nothing accepted, correction = first
    assert walk(build_trie([]), 5, 10, eos, lambda a, ch: 0) == ([], [], 5)


def _declared_symbols():
    text = (ROOT / "include" / "respect_b200.h").read_text()
    return sorted(set(re.findall(r"RB_API\s+[\w\s\*]+?\b(rb_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    from respect_b200 import _lib
    lib = _lib.lib()
    names = _declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert lib.rb_abi_version() == 1
    assert lib.rb_status_string(2) == b"unsupported shape, dtype or layout"


def test_capi_rejects_bad_arguments_without_a_gpu():
    """Host-side validation runs before any CUDA call: bad arguments return an
    error code (never reach a kernel)."""
    from respect_b200 import _lib
    lib = _lib.lib()
    assert lib.rb_linear(None, 8, None, 8, None, 8, _lib.RB_BF16, 1, 8, 8, None, 0, None) == 1
    assert lib.rb_silu_mul(None, None, None, 10, _lib.RB_BF16, None) == 1
    assert lib.rb_trie_node_mask(None, 4, 0, 2, 4, None, 4, None) == 1      # M < q
    args = _lib.AttnArgs()
    args.dtype, args.H, args.HK, args.D, args.M = _lib.RB_BF16, 28, 4, 64, 1   # head_dim 64 unsupported
    assert lib.rb_fused_attn_hyb(ctypes.byref(args), None, 0, None) in (1, 2)
    assert lib.rb_engine_workspace_bytes(None) == 0


def test_attention_rejects_node_rows_not_in_16_byte_units():
    """Node K/V rows are copied in 16-byte pieces: a bf16 row stride of 132
    elements (264 bytes) or a base off a 16-byte boundary is refused with
    RB_ERR_UNSUPPORTED before any CUDA call (the pointers here are never read)."""
    from respect_b200 import _lib
    lib = _lib.lib()

    def args(sknn=128, kn=0x100000, dtype=_lib.RB_BF16):
        a = _lib.AttnArgs()
        a.dtype, a.H, a.HK, a.D, a.M, a.NP, a.NN = dtype, 28, 4, 128, 16, 0, 32
        a.q, a.sqh, a.sqm, a.sqd = 0x200000, 16 * 128, 128, 1
        a.kn, a.sknh, a.sknn, a.sknd = kn, 32 * sknn, sknn, 1
        a.vn, a.svnh, a.svnn, a.svnd = 0x300000, 32 * 128, 128, 1
        a.msk, a.mask_kind, a.smm, a.smn = 0x400000, _lib.RB_MASK_BOOL, 32, 1
        a.out, a.soh, a.som, a.sod = 0x500000, 16 * 128, 128, 1
        a.sm_scale = 0.088
        return a

    for bad in (args(sknn=132), args(kn=0x100008), args(kn=0x100004)):
        assert lib.rb_fused_attn_hyb(ctypes.byref(bad), None, 0, None) == 2
    # the same call with 16-byte rows passes validation and only then asks for a workspace
    assert lib.rb_fused_attn_hyb(ctypes.byref(args()), None, 0, None) == 6


def test_engine_config_validation():
    from respect_b200.decoding import engine as E
    lib = __import__("respect_b200._lib", fromlist=["x"]).lib()
    fn = lib.rb_engine_workspace_bytes
    fn.restype, fn.argtypes = ctypes.c_size_t, [ctypes.POINTER(E._Cfg)]
    good = E._Cfg(3584, 28, 28, 4, 128, 18944, 152064, 1e-6, 128, 4096, 8192)
    assert fn(ctypes.byref(good)) > 0
    bad = E._Cfg(3584, 28, 28, 4, 64, 18944, 152064, 1e-6, 128, 4096, 8192)   # head_dim 64
    assert fn(ctypes.byref(bad)) == 0
    cfg = E.DecoderConfig.baseline_7b()
    # weights streamed per step: 6.525 G layer params + 0.545 G lm_head (bf16)
    assert abs(cfg.weight_bytes_per_step() / 1e9 - 14.14) < 0.01


def test_missing_library_fails_loudly(tmp_path):
    """Without the native library, loading it raises and so does every operator
    (CPU tensors are refused before that); nothing falls back to a CPU or library
    implementation."""
    import subprocess
    import sys
    code = (
        "import torch, respect_b200\n"
        "from respect_b200.kernels.rmsnorm import rmsnorm\n"
        "from respect_b200.system.fused import silu_mul\n"
        "try:\n"
        "    respect_b200.load()\n"
        "except ImportError as e:\n"
        "    assert 'no fallback' in str(e), e\n"
        "else:\n"
        "    raise SystemExit('loaded a library that is not there')\n"
        "for f, a in ((rmsnorm, (torch.ones(2, 8, dtype=torch.bfloat16), torch.ones(8, dtype=torch.bfloat16), 1e-6)),\n"
        "             (silu_mul, (torch.ones(4, dtype=torch.bfloat16), torch.ones(4, dtype=torch.bfloat16)))):\n"
        "    try:\n"
        "        f(*a)\n"
        "    except (ImportError, ValueError) as e:\n"
        "        assert 'no fallback' in str(e) or 'no CPU path' in str(e), e\n"
        "    else:\n"
        "        raise SystemExit('computed without the library')\n"
        "print('raised')\n")
    env = dict(__import__("os").environ, RESPECT_B200_LIB=str(tmp_path / "absent.so"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300,
                       cwd=str(__import__("pathlib").Path(__file__).resolve().parent.parent))
    assert r.returncode == 0 and "raised" in r.stdout, r.stdout + r.stderr
