"""ctypes binding of libultravec_b200.so (include/ultravec_b200.h).

The Python face of the C ABI, mirroring the reference's codec interface:
`Codec` is TrellisQuantizer's record API (src/trellis.rs:645-743) and
`Index` is its VectorBackend in codes-only mode (src/lib.rs:104-155,
src/trellis.rs:2088-2247).  Arrays may be numpy (host) or CUDA torch tensors
(device, ordered on torch's current stream); results come back in the same
kind.  There is no CPU fallback: a missing library or a CUDA failure raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libultravec_b200.so"

UV_OK, UV_EINVAL, UV_ENOMEM, UV_ECUDA, UV_ETIMEDOUT, UV_EUNSUPPORTED = range(6)
UV_SEARCH_COSINE, UV_SEARCH_MIPS = 0, 1

# Every symbol the header declares (checked by the CPU tests).
SYMBOLS = [
    "uv_abi_version", "uv_last_error", "uv_config_default", "uv_codec_create",
    "uv_codec_destroy", "uv_codec_code_table_bits", "uv_codec_rotation_sign_rounds",
    "uv_codec_memory_bits", "uv_codec_record_bytes", "uv_encode", "uv_encode_rotated",
    "uv_rotate", "uv_decode", "uv_windows", "uv_digest", "uv_index_create", "uv_index_destroy",
    "uv_index_set_centroids", "uv_index_reserve", "uv_index_add", "uv_index_add_batch",
    "uv_index_len", "uv_index_dimensions", "uv_index_mem_bytes", "uv_index_search",
    "uv_index_export", "uv_index_digest", "uv_index_clear", "uv_topk_merge",
    "uv_profile_enable", "uv_profile_read", "uv_set_tuning", "uv_index_search_noalloc",
    "uv_kmeans", "uv_ivf_assign", "uv_ivf_create", "uv_ivf_destroy", "uv_ivf_build",
    "uv_ivf_len", "uv_ivf_nlist", "uv_ivf_mem_bytes", "uv_ivf_probe", "uv_ivf_search", "uv_ivf_search_lists",
    "uv_ivf_search_rerank", "uv_ivf_export", "uv_ivf_digest", "uv_index_save", "uv_index_load",
    "uv_ivf_save", "uv_ivf_load", "uv_index_prepare", "uv_prepared_destroy", "uv_prepared_len",
    "uv_prepared_score", "uv_index_score_candidates", "uv_index_scorer_model_bytes",
    "uv_index_set_shortlist", "uv_index_export_signs", "uv_ivf_set_shortlist",
    "uv_ivf_export_signs", "uv_coset_create", "uv_coset_destroy", "uv_coset_set_centroids",
    "uv_coset_add", "uv_coset_search", "uv_coset_len", "uv_coset_shape", "uv_coset_books",
    "uv_coset_mem_bytes", "uv_coset_model_bytes", "uv_coset_export", "uv_coset_reconstruct",
    "uv_index_search_begin", "uv_search_set_bounds", "uv_search_finish", "uv_search_destroy",
    "uv_search_finish_deferred", "uv_search_check",
    "uv_topk_pack", "uv_topk_merge_packed", "uv_search_bounds_per_query", "uv_topk_unpack",
]


class UVError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ultravec_b200 error {code}: {msg}")
        self.code = code


class uv_config(C.Structure):
    _fields_ = [("dim", C.c_int32), ("bits", C.c_int32), ("mem", C.c_int32),
                ("rotation_rounds", C.c_int32), ("rotation_seed", C.c_uint64),
                ("start_bits", C.c_int32), ("rescale_bits", C.c_int32),
                ("branch_lambda", C.c_float), ("device", C.c_int32)]


_lib = None


def lib():
    """Load the in-tree library; fail loudly when it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `make -C {HERE}` (nvcc, sm_100a)")
        L = C.CDLL(str(LIB_PATH))
        vp, i32, i64, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64
        vpp = C.POINTER(C.c_void_p)
        sig = {
            "uv_abi_version": (C.c_int, []),
            "uv_last_error": (C.c_char_p, []),
            "uv_config_default": (None, [C.POINTER(uv_config), i32, i32, i32]),
            "uv_codec_create": (C.c_int, [C.POINTER(uv_config), vpp]),
            "uv_codec_destroy": (C.c_int, [vp]),
            "uv_codec_code_table_bits": (C.c_int, [vp, vp, i64]),
            "uv_codec_rotation_sign_rounds": (C.c_int, [vp, vp, i64]),
            "uv_codec_memory_bits": (C.c_int, [vp, C.POINTER(i32)]),
            "uv_codec_record_bytes": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32),
                                                C.POINTER(i32)]),
            "uv_encode": (C.c_int, [vp, vp, i64, vp, i32, vp, vp, vp, vp, vp, vp]),
            "uv_encode_rotated": (C.c_int, [vp, vp, i64, vp, vp, vp]),
            "uv_rotate": (C.c_int, [vp, vp, i64, vp, vp]),
            "uv_decode": (C.c_int, [vp, vp, vp, i64, vp, vp]),
            "uv_windows": (C.c_int, [vp, vp, vp, i64, vp, vp]),
            "uv_digest": (C.c_int, [vp, vp, vp, i64, C.POINTER(u64), vp]),
            "uv_index_create": (C.c_int, [vp, vpp]),
            "uv_index_destroy": (C.c_int, [vp]),
            "uv_index_set_centroids": (C.c_int, [vp, vp, i32]),
            "uv_index_reserve": (C.c_int, [vp, i64]),
            "uv_index_add": (C.c_int, [vp, vp, vp, i64, vp]),
            "uv_index_add_batch": (C.c_int, [vp, vp, i64, vp]),
            "uv_index_len": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_index_dimensions": (C.c_int, [vp, C.POINTER(i32)]),
            "uv_index_mem_bytes": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_index_search": (C.c_int, [vp, vp, i64, i32, i32, vp, vp, vp]),
            "uv_index_export": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, vp]),
            "uv_index_digest": (C.c_int, [vp, C.POINTER(u64), vp]),
            "uv_topk_merge": (C.c_int, [i32, vp, vp, i64, i32, i32, i32, vp, vp, vp]),
            "uv_index_clear": (C.c_int, [vp]),
            "uv_profile_enable": (C.c_int, [i32]),
            "uv_set_tuning": (C.c_int, [C.c_char_p, i64]),
            "uv_index_search_noalloc": (C.c_int, [vp, vp, i64, i32, i32, vp, vp, vp]),
            "uv_profile_read": (C.c_int, [C.c_char_p, C.POINTER(C.c_double), C.POINTER(i64)]),
            "uv_kmeans": (C.c_int, [i32, vp, i64, i32, i32, u64, i32, vp, vp]),
            "uv_ivf_assign": (C.c_int, [i32, vp, i64, i32, vp, i32, vp, vp]),
            "uv_ivf_create": (C.c_int, [vp, vp, i32, i32, vpp]),
            "uv_ivf_destroy": (C.c_int, [vp]),
            "uv_ivf_build": (C.c_int, [vp, vp, i64, vp, vp, vp]),
            "uv_ivf_len": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_ivf_nlist": (C.c_int, [vp, C.POINTER(i32)]),
            "uv_ivf_mem_bytes": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_ivf_probe": (C.c_int, [vp, vp, i64, i32, vp, vp]),
            "uv_ivf_search": (C.c_int, [vp, vp, i64, i32, i32, vp, vp, vp]),
            "uv_ivf_search_lists": (C.c_int, [vp, vp, i64, i32, i32, vp, vp, vp, vp]),
            "uv_ivf_search_rerank": (C.c_int, [vp, vp, i64, i32, i32, i32, vp, i64, vp, vp,
                                               vp]),
            "uv_ivf_export": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, vp]),
            "uv_ivf_digest": (C.c_int, [vp, C.POINTER(u64), vp]),
            "uv_index_save": (C.c_int, [vp, C.c_char_p]),
            "uv_index_load": (C.c_int, [vp, C.c_char_p, vpp]),
            "uv_ivf_save": (C.c_int, [vp, C.c_char_p]),
            "uv_ivf_load": (C.c_int, [vp, C.c_char_p, vpp]),
            "uv_index_prepare": (C.c_int, [vp, vp, i64, vpp, vp]),
            "uv_prepared_destroy": (C.c_int, [vp]),
            "uv_prepared_len": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_prepared_score": (C.c_int, [vp, vp, vp, i64, vp, vp]),
            "uv_index_score_candidates": (C.c_int, [vp, vp, vp, i64, vp, vp]),
            "uv_index_scorer_model_bytes": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_index_set_shortlist": (C.c_int, [vp, i32, i32, i32]),
            "uv_index_export_signs": (C.c_int, [vp, vp, vp]),
            "uv_ivf_set_shortlist": (C.c_int, [vp, i32, i32, i32]),
            "uv_ivf_export_signs": (C.c_int, [vp, vp, vp]),
            "uv_coset_create": (C.c_int, [i32, i32, i32, u64, i32, i32, vpp]),
            "uv_coset_destroy": (C.c_int, [vp]),
            "uv_coset_set_centroids": (C.c_int, [vp, vp, i32]),
            "uv_coset_add": (C.c_int, [vp, vp, vp, i64, vp]),
            "uv_coset_search": (C.c_int, [vp, vp, i64, i32, vp, vp, vp]),
            "uv_coset_len": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_coset_shape": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32)]),
            "uv_coset_books": (C.c_int, [vp, vp, vp]),
            "uv_coset_mem_bytes": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_coset_model_bytes": (C.c_int, [vp, C.POINTER(i64)]),
            "uv_coset_export": (C.c_int, [vp, vp, vp, vp, vp, vp, vp]),
            "uv_coset_reconstruct": (C.c_int, [vp, vp, i64, vp, vp]),
            "uv_index_search_begin": (C.c_int, [vp, vp, i64, i32, i32, i32, vp, vpp, vp]),
            "uv_search_set_bounds": (C.c_int, [vp, vp, i32]),
            "uv_search_finish": (C.c_int, [vp, vp, vp]),
            "uv_search_finish_deferred": (C.c_int, [vp, vp, vp]),
            "uv_search_check": (C.c_int, [vp, C.POINTER(C.c_int32)]),
            "uv_search_destroy": (C.c_int, [vp]),
            "uv_search_bounds_per_query": (C.c_int, [i32, i32, C.POINTER(i32)]),
            "uv_topk_pack": (C.c_int, [i32, vp, vp, i64, vp, vp]),
            "uv_topk_unpack": (C.c_int, [i32, vp, i64, vp, vp, vp]),
            "uv_topk_merge_packed": (C.c_int, [i32, vp, i64, i32, i32, i64, i64, i32, vp, vp,
                                               vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != UV_OK:
        raise UVError(rc, lib().uv_last_error().decode(errors="replace"))


# ---------------------------------------------------------------- arrays ---

def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


def _ptr(x):
    if x is None:
        return None
    if _is_torch(x):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return C.c_void_p(x.data_ptr())
    if not x.flags["C_CONTIGUOUS"]:
        raise ValueError("array must be C-contiguous")
    return C.c_void_p(x.ctypes.data)


def _stream(*arrays):
    for a in arrays:
        if a is not None and _is_torch(a) and a.is_cuda:
            import torch

            return C.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)
    return None


class _Alloc:
    """Output allocation in the same kind (numpy / torch-cuda) as an input.
    A pinned host tensor as input gives numpy outputs in pinned memory, so
    the library's device-to-host copies run at full speed."""

    def __init__(self, like):
        self.torch_dev = None
        self.pinned = False
        if like is not None and _is_torch(like):
            if like.is_cuda:
                self.torch_dev = like.device
            else:
                self.pinned = like.is_pinned()

    def __call__(self, shape, np_dtype):
        if self.torch_dev is None and not self.pinned:
            return np.zeros(shape, np_dtype)
        import torch

        tmap = {np.uint8: torch.uint8, np.uint32: torch.int32, np.float32: torch.float32,
                np.int64: torch.int64, np.int32: torch.int32}
        if self.pinned:
            t = torch.empty(shape, dtype=tmap[np_dtype], pin_memory=True)
            return t.numpy().view(np_dtype)
        return torch.zeros(shape, dtype=tmap[np_dtype], device=self.torch_dev)


def _i64(x):
    if _is_torch(x):
        import torch

        return x.to(torch.int64).contiguous()
    return np.ascontiguousarray(x, dtype=np.int64)


def _i32(x):
    if _is_torch(x):
        import torch

        return x.to(torch.int32).contiguous()
    return np.ascontiguousarray(x, dtype=np.int32)


def _f32(x):
    if _is_torch(x):
        import torch

        return x.to(torch.float32).contiguous()
    return np.ascontiguousarray(x, dtype=np.float32)


# ----------------------------------------------------------------- codec ---

class Codec:
    """TrellisQuantizer::from_config (src/trellis.rs:430-458) on one GPU."""

    def __init__(self, dim: int, bits: int, mem: int, *, seed: int = 42, rounds: int = 3,
                 start_bits: int | None = None, rescale_bits: int = 0,
                 branch_lambda: float = 0.0, device: int = 0):
        cfg = uv_config()
        lib().uv_config_default(C.byref(cfg), dim, bits, mem)
        cfg.rotation_seed = seed
        cfg.rotation_rounds = rounds
        cfg.start_bits = mem if start_bits is None else start_bits
        cfg.rescale_bits = rescale_bits
        cfg.branch_lambda = branch_lambda
        cfg.device = device
        h = C.c_void_p()
        check(lib().uv_codec_create(C.byref(cfg), C.byref(h)))
        self.h = h
        self.dim, self.bits, self.mem, self.device = dim, bits, mem, device
        self.rounds = max(1, rounds)
        cb, sb, rb = C.c_int32(), C.c_int32(), C.c_int32()
        check(lib().uv_codec_record_bytes(self.h, C.byref(cb), C.byref(sb), C.byref(rb)))
        self.code_bytes, self.start_bytes, self.rescale_bytes = cb.value, sb.value, rb.value

    def close(self):
        if getattr(self, "h", None):
            lib().uv_codec_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # record API -------------------------------------------------------
    def code_table_bits(self) -> np.ndarray:
        out = np.zeros(1 << (self.mem + self.bits), np.uint32)
        check(lib().uv_codec_code_table_bits(self.h, _ptr(out), out.size))
        return out

    def code_table(self) -> np.ndarray:
        return self.code_table_bits().view(np.float32)

    def rotation_sign_rounds(self) -> np.ndarray:
        out = np.zeros((self.rounds, self.dim), np.float32)
        check(lib().uv_codec_rotation_sign_rounds(self.h, _ptr(out), out.size))
        return out

    def memory_bits(self) -> int:
        m = C.c_int32()
        check(lib().uv_codec_memory_bits(self.h, C.byref(m)))
        return m.value

    def encode(self, rows, centroids=None):
        """encode_codes over a batch: dict(codes, start, rescale, rnorm, cidx)."""
        rows = _f32(rows)
        n = rows.shape[0]
        alloc = _Alloc(rows)
        out = dict(codes=alloc((n, self.code_bytes), np.uint8), start=alloc(n, np.uint32),
                   rescale=alloc(n, np.float32), rnorm=alloc(n, np.float32),
                   cidx=alloc(n, np.uint32))
        cen = None if centroids is None else _f32(centroids)
        ncen = 0 if cen is None else cen.shape[0]
        check(lib().uv_encode(self.h, _ptr(rows), n, _ptr(cen), ncen, _ptr(out["codes"]),
                              _ptr(out["start"]), _ptr(out["rescale"]), _ptr(out["rnorm"]),
                              _ptr(out["cidx"]), _stream(rows)))
        return out

    def encode_rotated(self, u_r):
        u_r = _f32(u_r)
        n = u_r.shape[0]
        alloc = _Alloc(u_r)
        codes, start = alloc((n, self.code_bytes), np.uint8), alloc(n, np.uint32)
        check(lib().uv_encode_rotated(self.h, _ptr(u_r), n, _ptr(codes), _ptr(start),
                                      _stream(u_r)))
        return codes, start

    def rotate(self, rows):
        rows = _f32(rows)
        out = _Alloc(rows)(rows.shape, np.float32)
        check(lib().uv_rotate(self.h, _ptr(rows), rows.shape[0], _ptr(out), _stream(rows)))
        return out

    def decode(self, codes, start):
        n = codes.shape[0]
        out = _Alloc(codes)((n, self.dim), np.float32)
        check(lib().uv_decode(self.h, _ptr(codes), _ptr(start), n, _ptr(out), _stream(codes)))
        return out

    def windows(self, codes, start):
        n = codes.shape[0]
        out = _Alloc(codes)((n, self.dim), np.uint32)
        check(lib().uv_windows(self.h, _ptr(codes), _ptr(start), n, _ptr(out), _stream(codes)))
        return out

    def digest(self, codes, start) -> int:
        h = C.c_uint64()
        check(lib().uv_digest(self.h, _ptr(codes), _ptr(start), codes.shape[0], C.byref(h),
                              _stream(codes)))
        return h.value


# ----------------------------------------------------------------- index ---

class Index:
    """Codes-only VectorBackend over the device-resident SoA records."""

    def __init__(self, codec: Codec):
        h = C.c_void_p()
        check(lib().uv_index_create(codec.h, C.byref(h)))
        self.h, self.codec = h, codec

    def close(self):
        if getattr(self, "h", None):
            lib().uv_index_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_centroids(self, centroids):
        cen = _f32(centroids)
        check(lib().uv_index_set_centroids(self.h, _ptr(cen), cen.shape[0]))

    def clear(self):
        check(lib().uv_index_clear(self.h))

    def reserve(self, additional: int):
        check(lib().uv_index_reserve(self.h, additional))

    def add(self, ids, rows):
        rows = _f32(rows)
        ids = ids if _is_torch(ids) else np.ascontiguousarray(ids, np.int64)
        check(lib().uv_index_add(self.h, _ptr(ids), _ptr(rows), rows.shape[0], _stream(rows)))

    def add_batch(self, rows):
        rows = _f32(rows)
        check(lib().uv_index_add_batch(self.h, _ptr(rows), rows.shape[0], _stream(rows)))

    def __len__(self) -> int:
        n = C.c_int64()
        check(lib().uv_index_len(self.h, C.byref(n)))
        return n.value

    def mem_bytes(self) -> int:
        n = C.c_int64()
        check(lib().uv_index_mem_bytes(self.h, C.byref(n)))
        return n.value

    def search(self, queries, k: int, mips: bool = False):
        """search (src/trellis.rs:2120-2183): top-k (ids, scores) per query."""
        queries = _f32(queries)
        nq = queries.shape[0]
        alloc = _Alloc(queries)
        ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
        check(lib().uv_index_search(self.h, _ptr(queries), nq, k,
                                    UV_SEARCH_MIPS if mips else UV_SEARCH_COSINE, _ptr(ids),
                                    _ptr(scores), _stream(queries)))
        return ids, scores

    def search_begin(self, queries, k: int, mips: bool = False, n_shards: int = 1):
        """Phase 1 of a search of this index as one shard of n_shards (see
        ShardSearch): query preparation and the prefilter's first pass."""
        return ShardSearch(self, queries, k, mips, n_shards)

    # -- the 1-bit shortlist (src/trellis.rs:803-948) --
    def set_shortlist(self, c: int, asym: bool = False, rnorm: bool = True) -> None:
        """with_shortlist(c).with_shortlist_asym(asym).with_shortlist_rnorm(rnorm);
        the index must be empty.  Cosine searches then run search_shortlist."""
        check(lib().uv_index_set_shortlist(self.h, c, int(asym), int(rnorm)))

    def export_signs(self):
        out = np.zeros((len(self), (self.codec.dim + 7) // 8), np.uint8)
        check(lib().uv_index_export_signs(self.h, _ptr(out), None))
        return out

    # -- CandidateScorer (src/lib.rs:93-102, src/trellis.rs:2039-2086) --
    def prepare(self, queries) -> "PreparedQueries":
        """CandidateScorer::prepare for a batch of queries (one row each)."""
        return PreparedQueries(self, queries)

    def score_candidates(self, query, positions):
        """prepare(query) then score_at(p) for every p in positions."""
        query = _f32(query).reshape(-1)
        positions = _i64(positions)
        out = _Alloc(positions)(positions.shape[0], np.float32)
        check(lib().uv_index_score_candidates(self.h, _ptr(query), _ptr(positions),
                                              positions.shape[0], _ptr(out),
                                              _stream(positions, query)))
        return out

    def scored_len(self) -> int:
        return len(self)

    def scorer_model_bytes(self) -> int:
        b = C.c_int64()
        check(lib().uv_index_scorer_model_bytes(self.h, C.byref(b)))
        return b.value

    def export(self):
        n = len(self)
        cb = self.codec.code_bytes
        out = dict(codes=np.zeros((n, cb), np.uint8), start=np.zeros(n, np.uint32),
                   rescale=np.zeros(n, np.float32), rnorm=np.zeros(n, np.float32),
                   norms=np.zeros(n, np.float32), ids=np.zeros(n, np.int64))
        check(lib().uv_index_export(self.h, _ptr(out["codes"]), _ptr(out["start"]),
                                    _ptr(out["rescale"]), _ptr(out["rnorm"]), _ptr(out["norms"]),
                                    _ptr(out["ids"]), None))
        return out

    def digest(self) -> int:
        h = C.c_uint64()
        check(lib().uv_index_digest(self.h, C.byref(h), None))
        return h.value

    def save(self, path) -> None:
        """Write the index file (records, sidecars, ids, centroids)."""
        check(lib().uv_index_save(self.h, os.fsencode(path)))

    @classmethod
    def load(cls, codec: Codec, path) -> "Index":
        """An index read from a file written by a codec of this configuration."""
        h = C.c_void_p()
        check(lib().uv_index_load(codec.h, os.fsencode(path), C.byref(h)))
        ix = cls.__new__(cls)
        ix.h, ix.codec = h, codec
        return ix


class CosetIndex:
    """The coset trellis backend (src/coset_trellis.rs, CosetTrellis): E8
    coset books, a 4-branch free-start Viterbi per row, and the same rescaled
    estimator.  dim % 8 == 0, bits 1..3; mem defaults to the reference's 12."""

    def __init__(self, dim: int, bits: int, mem: int = 12, seed: int = 42, rounds: int = 3,
                 device: int = 0):
        h = C.c_void_p()
        check(lib().uv_coset_create(dim, bits, mem, seed, rounds, device, C.byref(h)))
        self.h, self.dim, self.bits, self.mem, self.device = h, dim, bits, mem, device
        cl, pc = C.c_int32(), C.c_int32()
        check(lib().uv_coset_shape(h, C.byref(cl), C.byref(pc)))
        self.code_len, self.per_coset = cl.value, pc.value

    def close(self):
        if getattr(self, "h", None):
            lib().uv_coset_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_centroids(self, centroids):
        cen = _f32(centroids)
        check(lib().uv_coset_set_centroids(self.h, _ptr(cen), cen.shape[0]))

    def add(self, ids, rows):
        rows = _f32(rows)
        ids = ids if _is_torch(ids) else np.ascontiguousarray(ids, np.int64)
        check(lib().uv_coset_add(self.h, _ptr(ids), _ptr(rows), rows.shape[0], _stream(rows)))

    def add_batch(self, rows):
        """add_batch: ids are the batch's positions 0..n-1."""
        rows = _f32(rows)
        check(lib().uv_coset_add(self.h, None, _ptr(rows), rows.shape[0], _stream(rows)))

    def __len__(self) -> int:
        n = C.c_int64()
        check(lib().uv_coset_len(self.h, C.byref(n)))
        return n.value

    def mem_bytes(self) -> int:
        n = C.c_int64()
        check(lib().uv_coset_mem_bytes(self.h, C.byref(n)))
        return n.value

    def model_bytes(self) -> int:
        n = C.c_int64()
        check(lib().uv_coset_model_bytes(self.h, C.byref(n)))
        return n.value

    def search(self, queries, k: int):
        """search (src/coset_trellis.rs:471-497): top-k (ids, scores)."""
        queries = _f32(queries)
        nq = queries.shape[0]
        alloc = _Alloc(queries)
        ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
        check(lib().uv_coset_search(self.h, _ptr(queries), nq, k, _ptr(ids), _ptr(scores),
                                    _stream(queries)))
        return ids, scores

    def books(self):
        keys = np.zeros((8, self.per_coset), np.uint64)
        scale = np.zeros(2, np.float32)
        check(lib().uv_coset_books(self.h, _ptr(keys), _ptr(scale)))
        return keys, (float(scale[0]), float(scale[1]))

    def export(self):
        n = len(self)
        out = dict(codes=np.zeros((n, self.code_len), np.uint8), rescale=np.zeros(n, np.float32),
                   rnorm=np.zeros(n, np.float32), cidx=np.zeros(n, np.uint32),
                   ids=np.zeros(n, np.int64))
        check(lib().uv_coset_export(self.h, _ptr(out["codes"]), _ptr(out["rescale"]),
                                    _ptr(out["rnorm"]), _ptr(out["cidx"]), _ptr(out["ids"]),
                                    None))
        return out

    def reconstruct(self, rows):
        """reconstruct_unit of every row."""
        rows = _f32(rows)
        out = _Alloc(rows)(tuple(rows.shape), np.float32)
        check(lib().uv_coset_reconstruct(self.h, _ptr(rows), rows.shape[0], _ptr(out),
                                         _stream(rows)))
        return out


class PreparedQueries:
    """A batch of PreparedQuery (src/trellis.rs:2003-2037) on the index's GPU:
    score(positions, offsets) is score_at over CSR candidate lists."""

    def __init__(self, index: Index, queries):
        queries = _f32(queries)
        if queries.ndim == 1:
            queries = queries.reshape(1, -1)
        h = C.c_void_p()
        check(lib().uv_index_prepare(index.h, _ptr(queries), queries.shape[0], C.byref(h),
                                     _stream(queries)))
        self.h, self.index, self.nq = h, index, queries.shape[0]

    def close(self):
        if getattr(self, "h", None):
            check(lib().uv_prepared_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = C.c_int64()
        check(lib().uv_prepared_len(self.h, C.byref(n)))
        return n.value

    def score(self, positions, offsets=None):
        """Scores of positions[i] against query q for offsets[q] <= i < offsets[q+1]
        (all against the single query when offsets is None)."""
        positions = _i64(positions)
        off = None if offsets is None else _i64(offsets)
        out = _Alloc(positions)(positions.shape[0], np.float32)
        check(lib().uv_prepared_score(self.h, _ptr(off), _ptr(positions), positions.shape[0],
                                      _ptr(out), _stream(positions, off)))
        return out

    def score_at(self, position: int, query: int = 0) -> float:
        """One score_at call (a single-candidate batch)."""
        off = None
        if self.nq > 1:
            off = np.zeros(self.nq + 1, np.int64)
            off[query + 1:] = 1
        return float(self.score(np.array([position], np.int64), off)[0])


# ------------------------------------------------------------------- IVF ---

def kmeans(rows, nlist: int, seed: int = 42, iters: int = 5, device: int = 0):
    """bench.rs:298-349 k-means of the unit-normalized rows (nlist x dim)."""
    rows = _f32(rows)
    out = _Alloc(rows)((nlist, rows.shape[1]), np.float32)
    check(lib().uv_kmeans(device, _ptr(rows), rows.shape[0], rows.shape[1], nlist, seed, iters,
                          _ptr(out), _stream(rows)))
    return out


def ivf_assign(rows, centroids, device: int = 0):
    """ivf.rs:405-421: first strict maximum of <row / |row|, c_j>."""
    rows, cen = _f32(rows), _f32(centroids)
    out = _Alloc(rows)((rows.shape[0],), np.uint32)
    check(lib().uv_ivf_assign(device, _ptr(rows), rows.shape[0], rows.shape[1], _ptr(cen),
                              cen.shape[0], _ptr(out), _stream(rows)))
    return out


class IvfIndex:
    """IvfIndex (ivf.rs:155-274) over one codec: centroids + posting lists."""

    def __init__(self, codec: Codec, centroids, centered: bool = False):
        cen = _f32(centroids)
        h = C.c_void_p()
        check(lib().uv_ivf_create(codec.h, _ptr(cen), cen.shape[0], 1 if centered else 0,
                                  C.byref(h)))
        self.h, self.codec, self.centered = h, codec, centered

    def close(self):
        if getattr(self, "h", None):
            lib().uv_ivf_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def build(self, rows, assign=None, ids=None):
        """IvfIndex::build (ivf.rs:171-205); assign None computes it."""
        rows = _f32(rows)
        if assign is not None and not _is_torch(assign):
            assign = np.ascontiguousarray(assign, np.uint32)
        if ids is not None and not _is_torch(ids):
            ids = np.ascontiguousarray(ids, np.int64)
        check(lib().uv_ivf_build(self.h, _ptr(rows), rows.shape[0], _ptr(assign), _ptr(ids),
                                 _stream(rows)))

    def __len__(self) -> int:
        n = C.c_int64()
        check(lib().uv_ivf_len(self.h, C.byref(n)))
        return n.value

    @property
    def nlist(self) -> int:
        n = C.c_int32()
        check(lib().uv_ivf_nlist(self.h, C.byref(n)))
        return n.value

    def mem_bytes(self) -> int:
        n = C.c_int64()
        check(lib().uv_ivf_mem_bytes(self.h, C.byref(n)))
        return n.value

    def probe(self, queries, nprobe: int):
        queries = _f32(queries)
        out = _Alloc(queries)((queries.shape[0], nprobe), np.int32)
        check(lib().uv_ivf_probe(self.h, _ptr(queries), queries.shape[0], nprobe, _ptr(out),
                                 _stream(queries)))
        return out

    def set_shortlist(self, c: int, asym: bool = False, rnorm: bool = True) -> None:
        """IvfCodec::TrellisShortlist{c, asym, rnorm} (ivf.rs:52-60); before build."""
        check(lib().uv_ivf_set_shortlist(self.h, c, int(asym), int(rnorm)))

    def export_signs(self):
        out = np.zeros((len(self), (self.codec.dim + 7) // 8), np.uint8)
        check(lib().uv_ivf_export_signs(self.h, _ptr(out), None))
        return out

    def search(self, queries, k: int, nprobe: int):
        """search (ivf.rs:229-239): top-k (ids, scores) per query."""
        queries = _f32(queries)
        nq = queries.shape[0]
        alloc = _Alloc(queries)
        ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
        check(lib().uv_ivf_search(self.h, _ptr(queries), nq, k, nprobe, _ptr(ids), _ptr(scores),
                                  _stream(queries)))
        return ids, scores

    def search_lists(self, queries, k: int, lists):
        """search over probe lists chosen beforehand (nq x nprobe, -1 = no
        list), e.g. by another shard's probe with the same centroids."""
        queries, lists = _f32(queries), _i32(lists)
        nq, nprobe = queries.shape[0], lists.shape[1]
        alloc = _Alloc(queries)
        ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
        check(lib().uv_ivf_search_lists(self.h, _ptr(queries), nq, k, nprobe, _ptr(lists),
                                        _ptr(ids), _ptr(scores), _stream(queries)))
        return ids, scores

    def search_with_rerank(self, queries, k: int, nprobe: int, rdepth: int, db):
        """search_with_rerank (ivf.rs:248-274): exact fp32 cosine of the top-rdepth."""
        queries, db = _f32(queries), _f32(db)
        nq = queries.shape[0]
        alloc = _Alloc(queries)
        ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
        check(lib().uv_ivf_search_rerank(self.h, _ptr(queries), nq, k, nprobe, rdepth, _ptr(db),
                                         db.shape[0], _ptr(ids), _ptr(scores),
                                         _stream(queries)))
        return ids, scores

    def export(self):
        n, cb = len(self), self.codec.code_bytes
        out = dict(list_off=np.zeros(self.nlist + 1, np.int64), ids=np.zeros(n, np.int64),
                   codes=np.zeros((n, cb), np.uint8), start=np.zeros(n, np.uint32),
                   rescale=np.zeros(n, np.float32), rnorm=np.zeros(n, np.float32))
        check(lib().uv_ivf_export(self.h, _ptr(out["list_off"]), _ptr(out["ids"]),
                                  _ptr(out["codes"]), _ptr(out["start"]), _ptr(out["rescale"]),
                                  _ptr(out["rnorm"]), None))
        return out

    def digest(self) -> int:
        h = C.c_uint64()
        check(lib().uv_ivf_digest(self.h, C.byref(h), None))
        return h.value

    def save(self, path) -> None:
        check(lib().uv_ivf_save(self.h, os.fsencode(path)))

    @classmethod
    def load(cls, codec: Codec, path) -> "IvfIndex":
        h = C.c_void_p()
        check(lib().uv_ivf_load(codec.h, os.fsencode(path), C.byref(h)))
        ix = cls.__new__(cls)
        ix.h, ix.codec, ix.centered = h, codec, None
        return ix


class ShardSearch:
    """A search of one shard of a base split across GPUs
    (uv_index_search_begin / uv_search_set_bounds / uv_search_finish):
    `bounds` (nq x m) are this shard's best first-pass lower bounds; gather
    every shard's bounds shard-major into (n_shards * nq, m), pass them to
    set_bounds, then finish() gives this shard's (ids, scores), at most k per
    query, of which only records that can be in the global top k remain."""

    def __init__(self, index: Index, queries, k: int, mips: bool, n_shards: int):
        queries = _f32(queries)
        self.nq, self.k = queries.shape[0], k
        self._alloc = _Alloc(queries)
        m = C.c_int32()
        check(lib().uv_search_bounds_per_query(k, n_shards, C.byref(m)))
        self.m = m.value
        self.bounds = self._alloc((self.nq, self.m), np.float32)
        h = C.c_void_p()
        check(lib().uv_index_search_begin(index.h, _ptr(queries), self.nq, k,
                                          UV_SEARCH_MIPS if mips else UV_SEARCH_COSINE,
                                          n_shards, _ptr(self.bounds), C.byref(h),
                                          _stream(queries)))
        self.h, self.index = h, index

    def set_bounds(self, gathered, n_shards: int):
        gathered = _f32(gathered)
        check(lib().uv_search_set_bounds(self.h, _ptr(gathered), n_shards))

    def finish(self, deferred: bool = False):
        """This shard's (ids, scores).  deferred (device queries only): the
        work is queued and the call returns at once; the lists are final
        after check()."""
        ids = self._alloc((self.nq, self.k), np.int64)
        scores = self._alloc((self.nq, self.k), np.float32)
        fn = (lib().uv_search_finish_deferred if deferred and _is_torch(ids) and ids.is_cuda
              else lib().uv_search_finish)
        check(fn(self.h, _ptr(ids), _ptr(scores)))
        return ids, scores

    def check(self) -> bool:
        """Waits for the search; True when some query overflowed the
        prefilter and was rescanned exactly (its slots rewritten in the lists
        finish returned, which must then be merged again)."""
        over = C.c_int32()
        check(lib().uv_search_check(self.h, C.byref(over)))
        return bool(over.value)

    def close(self):
        if getattr(self, "h", None):
            lib().uv_search_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def topk_pack(ids, scores, device: int = 0, out=None):
    """(nq, k) device ids and scores as one (nq, k, 3) int32 tensor of
    12-byte records (id low, id high, score bits): one buffer per collective.
    `out` (contiguous, nq * k * 3 int32) receives them when given."""
    import torch

    if out is None:
        out = torch.empty(tuple(ids.shape) + (3,), dtype=torch.int32, device=ids.device)
    check(lib().uv_topk_pack(device, _ptr(ids), _ptr(scores), ids.numel(), _ptr(out),
                             _stream(ids)))
    return out


def topk_unpack(packed, device: int = 0):
    """Inverse of topk_pack: (..., 3) int32 device records -> ids, scores."""
    import torch

    shape = tuple(packed.shape[:-1])
    ids = torch.empty(shape, dtype=torch.int64, device=packed.device)
    scores = torch.empty(shape, dtype=torch.float32, device=packed.device)
    check(lib().uv_topk_unpack(device, _ptr(packed.contiguous()), ids.numel(), _ptr(ids),
                               _ptr(scores), _stream(packed)))
    return ids, scores


def topk_merge_packed(packed, nq: int, n_lists: int, k_in: int, k: int, row_stride: int = 0,
                      list_stride: int = 0, device: int = 0):
    """Merge packed per-shard lists: list l of row q starts at record
    q * row_stride + l * list_stride (0, 0: contiguous rows)."""
    alloc = _Alloc(packed)
    ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
    check(lib().uv_topk_merge_packed(device, _ptr(packed), nq, n_lists, k_in, row_stride,
                                     list_stride, k, _ptr(ids), _ptr(scores), _stream(packed)))
    return ids, scores


def topk_merge(in_ids, in_scores, k: int, device: int = 0):
    """Merge per-shard top-k lists: in_* are nq x n_lists x k_in."""
    nq, n_lists, k_in = in_ids.shape
    alloc = _Alloc(in_ids)
    ids, scores = alloc((nq, k), np.int64), alloc((nq, k), np.float32)
    check(lib().uv_topk_merge(device, _ptr(in_ids), _ptr(in_scores), nq, n_lists, k_in, k,
                              _ptr(ids), _ptr(scores), _stream(in_ids)))
    return ids, scores


def set_tuning(key: str, value: int):
    """Launch-shape tuning (never changes results), e.g. ("scan_splits", 8)."""
    check(lib().uv_set_tuning(key.encode(), int(value)))


def profile_enable(on: bool = True):
    check(lib().uv_profile_enable(1 if on else 0))


def profile_read(kernel: str = "*"):
    """(total device ms, launches) of one kernel family since profile_enable."""
    ms, n = C.c_double(), C.c_int64()
    check(lib().uv_profile_read(kernel.encode(), C.byref(ms), C.byref(n)))
    return ms.value, n.value


def build(verbose: bool = False) -> Path:
    """Compile the library for sm_100a with the package Makefile."""
    import subprocess

    cmd = ["make", "-C", str(HERE), f"-j{min(8, os.cpu_count() or 1)}"]
    subprocess.run(cmd, check=True, capture_output=not verbose)
    return LIB_PATH
