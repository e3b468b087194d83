"""CPU checks of the C-ABI boundary: the library loads without a GPU, exports every
symbol declared in include/gsplat_b200.h, the ctypes signatures match the header,
and argument validation fails loudly (no kernel is launched in these tests)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gsplat_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return re.findall(r"GSB_API\s+[\w\s\*]+?\b(gsb_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 20
    for n in ("gsb_projection_fused_fwd", "gsb_projection_fused_bwd", "gsb_isect_emit",
              "gsb_radix_sort_pairs", "gsb_rasterize_fwd", "gsb_rasterize_bwd", "gsb_adam"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from gsplat_b200.cuda import _backend

    lib = _backend.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_signatures_cover_header():
    from gsplat_b200.cuda import _backend

    declared = set(declared_functions())
    assert declared == set(_backend.SIGNATURES), declared ^ set(_backend.SIGNATURES)
    text = open(HEADER).read()
    for name, (_, args) in _backend.SIGNATURES.items():
        m = re.search(r"GSB_API[^;(]*\b" + name + r"\s*\(([^;]*)\)\s*;", text, re.S)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))


def test_invalid_arguments_return_errors_without_launch():
    from gsplat_b200.cuda import _backend

    lib = _backend.lib()
    assert lib.gsb_version() == 1
    rc = lib.gsb_spherical_harmonics_fwd(7, 10, 64, None, None, None, None, None)
    assert rc == -2 and b"degree" in lib.gsb_last_error()
    rc = lib.gsb_rasterize_fwd(1, 0, None, None, None, None, None, None, 16, 16, 16, 1, 1, None,
                               None, 0, None, None, None, None)
    assert rc == -1 and b"channels" in lib.gsb_last_error()
    rc = lib.gsb_isect_count(0, 1 << 20, 1, 0, None, None, None, None, None, None, 16, 4096, 4096,
                             None, None)
    assert rc == -1 and b"exceed" in lib.gsb_last_error()
    rc = lib.gsb_projection_fused_fwd(1, 1, 1, None, None, None, None, None, None, None, 1, 1, 0.3,
                                      0.01, 100.0, 0.0, 0, 3, None, None, None, None, None, None)
    assert rc == -2 and b"camera_model" in lib.gsb_last_error()
    rc = lib.gsb_proj_fwd(1, 1, 1, None, None, None, 1, 1, 4, None, None, None)
    assert rc == -2 and b"camera_model" in lib.gsb_last_error()
    rc = lib.gsb_quat_scale_to_covar_preci_fwd(-1, None, None, 0, None, None, None)
    assert rc == -1 and b"negative" in lib.gsb_last_error()
    rc = lib.gsb_adam_multi(2, None, None, 0.9, 0.999, None)
    assert rc == -1 and b"no group list" in lib.gsb_last_error()
    assert lib.gsb_adam_multi(0, None, None, 0.9, 0.999, None) == 0  # nothing to do, nothing launched


def test_peer_exchange_arguments_checked_before_any_cuda_call():
    """The peer-memory exchange entry points reject a missing or inconsistent
    group, missing array lists and exchange number 0 before touching the
    device."""
    import ctypes

    from gsplat_b200.cuda import _backend

    lib = _backend.lib()
    assert lib.gsb_peer_mailbox_bytes() >= 4096
    assert lib.gsb_peer_open(None, None) == -1 and b"peer open" in lib.gsb_last_error()
    assert lib.gsb_peer_error_alloc(None, None) == -1 and b"error word" in lib.gsb_last_error()
    assert lib.gsb_peer_alloc(0, None, None) == -1
    w = (ctypes.c_int * 1)(2)
    srcs = (ctypes.c_void_p * 1)(None)
    rc = lib.gsb_peer_send_rows(None, 1, 0, None, None, None, 1, 0, 1, srcs, w, None)
    assert rc == -1 and b"rank / world" in lib.gsb_last_error()
    g = _backend.GsbPeerGroup()
    g.rank, g.world = 0, 2  # arenas not mapped
    rc = lib.gsb_peer_recv_rows(ctypes.byref(g), 1, 0, None, None, None, 1, 0, 1, srcs, w, None)
    assert rc == -1 and b"not mapped" in lib.gsb_last_error()
    g.world = 1
    g.arena[0] = 4096  # never dereferenced: the checks below fail first
    rc = lib.gsb_peer_send_grads(ctypes.byref(g), 1, 0, None, None, 0, 1, srcs, w, None)
    assert rc == -1 and b"error word" in lib.gsb_last_error()
    g.error = 8192
    rc = lib.gsb_peer_recv_grads(ctypes.byref(g), 1, 0, None, 1, None, None, None)
    assert rc == -1 and b"no array list" in lib.gsb_last_error()
    rc = lib.gsb_peer_recv_grads(ctypes.byref(g), 0, 0, None, 1, srcs, w, None)
    assert rc == -1 and b"peer recv grads" in lib.gsb_last_error()
    rc = lib.gsb_pack_rows(4, None, 1, None, None, None, None)
    assert rc == -1 and b"no array list" in lib.gsb_last_error()


def test_python_ops_raise_on_cpu_tensors():
    import torch

    import gsplat_b200

    with pytest.raises(RuntimeError, match="CUDA tensor"):
        gsplat_b200.spherical_harmonics(1, torch.randn(4, 3), torch.randn(4, 4, 3))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        gsplat_b200.fully_fused_projection(torch.randn(4, 3), None, torch.randn(4, 4),
                                           torch.rand(4, 3), torch.eye(4)[None], torch.eye(3)[None],
                                           8, 8)


def test_api_signature_matches_reference():
    """Keyword names and defaults of the drop-in API (reference rendering.py:256-310,
    _wrapper.py:479-497, 634-651, 829-843)."""
    import inspect

    import gsplat_b200

    sig = inspect.signature(gsplat_b200.rasterization)
    defaults = {k: v.default for k, v in sig.parameters.items()}
    expect = dict(near_plane=0.01, far_plane=1e10, radius_clip=0.0, eps2d=0.3, sh_degree=None,
                  packed=True, tile_size=16, backgrounds=None, render_mode="RGB",
                  sparse_grad=False, absgrad=False, rasterize_mode="classic", channel_chunk=32,
                  distributed=False, camera_model="pinhole", segmented=False, covars=None)
    for k, v in expect.items():
        assert defaults[k] == v, k
    params = list(sig.parameters)
    assert params[:9] == ["means", "quats", "scales", "opacities", "colors", "viewmats", "Ks",
                          "width", "height"]
    p = list(inspect.signature(gsplat_b200.fully_fused_projection).parameters)
    assert p == ["means", "covars", "quats", "scales", "viewmats", "Ks", "width", "height", "eps2d",
                 "near_plane", "far_plane", "radius_clip", "packed", "sparse_grad",
                 "calc_compensations", "camera_model", "opacities"]
    p = list(inspect.signature(gsplat_b200.isect_tiles).parameters)
    assert p == ["means2d", "radii", "depths", "tile_size", "tile_width", "tile_height", "sort",
                 "segmented", "packed", "n_images", "image_ids", "gaussian_ids", "conics",
                 "opacities"]
    p = list(inspect.signature(gsplat_b200.rasterize_to_pixels).parameters)
    assert p == ["means2d", "conics", "colors", "opacities", "image_width", "image_height",
                 "tile_size", "isect_offsets", "flatten_ids", "backgrounds", "masks", "packed",
                 "absgrad"]


def test_bucket_shard_plan():
    """Few buckets: one shard per CTA of the shared-memory path; many buckets:
    the GSB_ISECT_BUCKET_SHARDS global shards of the header."""
    from gsplat_b200.cuda import _backend

    text = open(HEADER).read()
    m = re.search(r"#define GSB_ISECT_BUCKET_SHARDS (\d+)", text)
    lib = _backend.lib()
    assert lib.gsb_isect_bucket_shards(1, 2000, 2000) == int(m.group(1))
    assert lib.gsb_isect_bucket_shards(1, 81, 53) >= 32


def declared_arities():
    """Parameter count of every GSB_API prototype in the header."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"GSB_API\s+[\w\s\*]+?\b(gsb_\w+)\s*\((.*?)\)\s*;", text, flags=re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_argument_counts_match_header():
    from gsplat_b200.cuda import _backend

    arity = declared_arities()
    assert len(arity) == len(declared_functions())
    wrong = {n: (arity[n], len(_backend.SIGNATURES[n][1])) for n in arity
             if len(_backend.SIGNATURES[n][1]) != arity[n]}
    assert not wrong, wrong


def _ctype_of(param: str):
    """ctypes type a header parameter declaration maps to."""
    import ctypes

    p = " ".join(param.split())
    if "*" in p or p.startswith("cudaStream_t"):
        return ctypes.c_void_p
    base = p.rsplit(" ", 1)[0] if " " in p else p
    base = base.replace("const ", "")
    return {"int": ctypes.c_int, "long long": ctypes.c_longlong, "float": ctypes.c_float,
            "size_t": ctypes.c_size_t, "unsigned long long": ctypes.c_ulonglong,
            "bool": ctypes.c_bool}[base]


def test_ctypes_argument_types_match_header():
    import ctypes

    from gsplat_b200.cuda import _backend

    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    wrong = []
    for m in re.finditer(r"GSB_API\s+[\w\s\*]+?\b(gsb_\w+)\s*\((.*?)\)\s*;", text, flags=re.S):
        name, params = m.group(1), m.group(2).strip()
        if params in ("", "void"):
            continue
        want = [_ctype_of(q) for q in params.split(",")]
        have = _backend.SIGNATURES[name][1]
        # structure / array pointers are bound as pointers too
        have = [ctypes.c_void_p if (isinstance(h, type) and issubclass(h, ctypes._Pointer)) else h for h in have]
        if [w.__name__ for w in want] != [getattr(h, "__name__", str(h)) for h in have]:
            wrong.append((name, [w.__name__ for w in want], [getattr(h, "__name__", str(h)) for h in have]))
    assert not wrong, wrong[:3]
