"""CPU checks of the C-ABI library: it loads without a GPU and exports every entry point that
include/b200_paged.h declares (no compute calls)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", fn)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", src, flags=re.M):
            name = m.group(1)
            if name not in ("if", "while", "for", "return", "sizeof", "defined"):
                names.add(name)
    return names


def test_library_exports_every_declared_symbol(pkg):
    from llm_serving_b200 import _native
    lib = ctypes.CDLL(_native.LIB_PATH)
    declared = _declared()
    assert "paged_attention" in declared and "b200_paged_decode" in declared
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes binding covers the same set
    assert declared == set(_native.exported_symbols())
    _native.lib()  # binds every signature


def test_status_strings(pkg):
    from llm_serving_b200 import _native
    L = _native.lib()
    assert L.b200_status_string(0) == b"ok"
    assert L.b200_status_string(2) == b"out of memory"


def _decode_workspace_layout(S, max_ctx, split, hkv=8, G=4, D=128):
    """The decode workspace layout (header, split offsets, work list, merge counters, partial
    lse and o) for a given split length, restated from the library's plan."""
    a256 = lambda x: (x + 255) & ~255
    ips = hkv * ((G + 7) // 8)
    hpc = min(G, 8)
    ms = S * ((max_ctx + split - 1) // split)
    return (a256(16) + a256((S + 1) * 4) + a256(ms * 8) + a256(S * ips * 4) + a256(ms * ips * hpc * 4)
            + a256(ms * ips * hpc * D * 4))


def test_decode_split_rule_on_host(pkg):
    """Pins the split rule through the workspace size (host arithmetic, no GPU needed; without a
    device the library plans for 148 SMs): 2048-token splits, halved down to 512 while there are
    fewer (sequence, split, kv head) items than half the SMs."""
    from llm_serving_b200 import _native as N
    L = N.lib()

    def ws(S, max_ctx):
        p = N.DecodeParams()
        p.geom = N.CacheGeometry(1, 1024, 16, 8, 128, N.DTYPE_BF16)
        p.num_query_heads, p.num_seqs, p.max_context_len = 32, S, max_ctx
        p.q_stride_row, p.q_stride_head = 32 * 128, 128
        return int(L.b200_paged_decode_workspace_bytes(ctypes.byref(p)))

    # config 2: 256 sequences, contexts up to 4096 -> 2048-token splits
    assert ws(256, 4096) == _decode_workspace_layout(256, 4096, 2048)
    assert ws(256, 4096) != _decode_workspace_layout(256, 4096, 4096)
    # a long-context batch of 14 sequences, and a single 32k sequence (128 items) -> 2048
    assert ws(14, 33792) == _decode_workspace_layout(14, 33792, 2048)
    assert ws(1, 32768) == _decode_workspace_layout(1, 32768, 2048)
    # two sequences of 4096 give 32 items at 2048 -> 1024 (64 items) -> 512 (128 items)
    assert ws(2, 4096) == _decode_workspace_layout(2, 4096, 512)
    # a tiny batch bottoms out at 512
    assert ws(4, 700) == _decode_workspace_layout(4, 700, 512)
