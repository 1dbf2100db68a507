"""ctypes view of the CPU oracle (oracle/liboracle_uv.so).

TEST INFRASTRUCTURE ONLY: the checker that the CUDA path is compared against
and the timed CPU baseline.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg; never by the product package.

Each wrapper names the reference function it restates (ultravec-ann sources).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_uv.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i16p = np.ctypeslib.ndpointer(np.int16, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_vp = C.c_void_p


def build() -> Path:
    """Compile the oracle with its Makefile (gcc is enough; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sig = {
            "uvo_inv_norm_cdf": (C.c_double, [C.c_double]),
            "uvo_gaussian_code": (C.c_float, [C.c_uint32]),
            "uvo_l2_norm": (C.c_float, [_f32p, C.c_int]),
            "uvo_l2_norms": (None, [_f32p, C.c_int64, C.c_int, _f32p, C.c_int]),
            "uvo_std_about_mean": (C.c_float, [_f32p, C.c_int]),
            "uvo_fwht": (None, [_f32p, C.c_int]),
            "uvo_pack_indices": (C.c_int, [_u16p, C.c_int, C.c_int, _u8p]),
            "uvo_unpack_indices": (None, [_u8p, C.c_int, C.c_int, _u16p, C.c_int]),
            "uvo_lut_dot_u32": (C.c_float, [_f32p, _u32p, _f32p, C.c_int]),
            "uvo_dense_dot": (C.c_float, [_f32p, _f32p, C.c_int]),
            "uvo_acs_step": (None, [_f32p, _f32p, C.c_int, C.c_int, _f32p, _u8p]),
            "uvo_codec_new": (_vp, [C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int, C.c_int,
                                    C.c_int, C.c_float]),
            "uvo_codec_free": (None, [_vp]),
            "uvo_e8_key": (C.c_uint64, [_i16p]),
            "uvo_e8_unkey": (None, [C.c_uint64, _i16p]),
            "uvo_coset_of": (C.c_int, [_i16p]),
            "uvo_e8_nearest": (None, [_f32p, _f32p]),
            "uvo_e8_enumerate": (C.c_int64, [C.c_float, _vp, C.c_int64]),
            "uvo_coset_new": (_vp, [C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int]),
            "uvo_coset_free": (None, [_vp]),
            "uvo_coset_set_centroids": (C.c_int, [_vp, _f32p, C.c_int]),
            "uvo_coset_per_coset": (C.c_int, [_vp]),
            "uvo_coset_code_len": (C.c_int, [_vp]),
            "uvo_coset_books": (None, [_vp, _u64p]),
            "uvo_coset_scale": (None, [_vp, _f32p]),
            "uvo_coset_index": (C.c_int64, [_vp, C.c_int, _i16p]),
            "uvo_coset_nearest": (None, [_vp, C.c_int, _f32p, C.POINTER(C.c_int64),
                                         C.POINTER(C.c_float)]),
            "uvo_coset_nearest_exhaustive": (None, [_vp, C.c_int, _f32p, C.POINTER(C.c_int64),
                                                    C.POINTER(C.c_float)]),
            "uvo_coset_encode_batch": (None, [_vp, _f32p, C.c_int64, _u8p, _f32p, _f32p, _u32p]),
            "uvo_coset_decode": (None, [_vp, _u8p, _f32p]),
            "uvo_coset_reconstruct_unit": (None, [_vp, _f32p, _f32p]),
            "uvo_coset_search": (None, [_vp, _u8p, _f32p, _f32p, _u32p, _vp, C.c_int64, _f32p,
                                        C.c_int64, C.c_int, _i64p, _f32p]),
            "uvo_coset_mem_bytes": (C.c_int64, [_vp, C.c_int64]),
            "uvo_codec_set_centroids": (C.c_int, [_vp, _f32p, C.c_int]),
            "uvo_codec_code_bytes": (C.c_int, [_vp]),
            "uvo_codec_table_len": (C.c_int, [_vp]),
            "uvo_codec_table": (None, [_vp, _f32p]),
            "uvo_codec_signs": (None, [_vp, _f32p]),
            "uvo_rotate": (None, [_vp, _f32p, _f32p]),
            "uvo_rotate_inverse": (None, [_vp, _f32p, _f32p]),
            "uvo_encode": (C.c_int, [_vp, _f32p, _u8p, _u32p, _f32p, _f32p, _u32p]),
            "uvo_encode_scalar_ref": (C.c_int, [_vp, _f32p, _u8p, _u32p]),
            "uvo_encode_rotated": (C.c_int, [_vp, _f32p, _u8p, _u32p]),
            "uvo_encode_batch": (None, [_vp, _f32p, C.c_int64, _u8p, _u32p, _f32p, _f32p,
                                        _u32p, C.c_int]),
            "uvo_digest": (C.c_uint64, [_u8p, _u32p, C.c_int64, C.c_int]),
            "uvo_windows": (None, [_vp, _u8p, C.c_uint32, _u32p]),
            "uvo_window_at": (C.c_uint32, [_vp, _u8p, C.c_uint32, C.c_int]),
            "uvo_decode_codes": (None, [_vp, _u8p, C.c_uint32, _f32p]),
            "uvo_reconstruct_unit": (None, [_vp, _u8p, C.c_uint32, C.c_float, C.c_uint32,
                                            _f32p]),
            "uvo_prepare_query": (C.c_int, [_vp, _f32p, _f32p, _f32p]),
            "uvo_score": (C.c_float, [_vp, _f32p, C.c_float, _u8p, C.c_uint32, C.c_float,
                                      C.c_float]),
            "uvo_search_topk": (None, [_vp, _u8p, _u32p, _f32p, _vp, _vp, _vp, C.c_int64,
                                       _f32p, C.c_int64, C.c_int, _i64p, _f32p, C.c_int]),
            "uvo_encode_batch_signs": (None, [_vp, _f32p, C.c_int64, _u8p, _u32p, _f32p, _f32p,
                                              _u32p, _u8p, C.c_int]),
            "uvo_ivf_encode_signs": (None, [_vp, _f32p, C.c_int64, _vp, _u32p, _u8p, _u32p,
                                            _f32p, _f32p, _u8p, C.c_int]),
            "uvo_search_shortlist": (None, [_vp, _u8p, _u32p, _f32p, _vp, _vp, _u8p, C.c_int64,
                                            _f32p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int,
                                            _i64p, _f32p, C.c_int]),
            "uvo_ivf_search_shortlist": (None, [_vp, _f32p, C.c_int, _i64p, _i64p, _u8p, _u32p,
                                                _f32p, _f32p, _u8p, C.c_int, _f32p, C.c_int64,
                                                C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                _i64p, _f32p, C.c_int]),
            "uvo_score_candidates": (None, [_vp, _u8p, _u32p, _f32p, _vp, _vp, _f32p, C.c_int64,
                                            _vp, _i64p, C.c_int64, _f32p, C.c_int]),
            "uvo_exact_topk": (None,[_f32p, C.c_int64, C.c_int, _f32p, C.c_int64, C.c_int,
                                      C.c_int, _i64p, C.c_int]),
            "uvo_kmeans": (None, [_f32p, C.c_int64, C.c_int, C.c_int, C.c_uint64, C.c_int,
                                  _f32p, C.c_int]),
            "uvo_assign": (None, [_f32p, C.c_int64, C.c_int, _f32p, C.c_int, _u32p, C.c_int]),
            "uvo_ivf_probe": (None, [_f32p, C.c_int, C.c_int, _f32p, C.c_int, _i32p]),
            "uvo_ivf_encode": (None, [_vp, _f32p, C.c_int64, _vp, _u32p, _u8p, _u32p, _f32p,
                                      _f32p, C.c_int]),
            "uvo_ivf_search_topk": (None, [_vp, _f32p, C.c_int, _i64p, _i64p, _u8p, _u32p,
                                           _f32p, _f32p, C.c_int, _f32p, C.c_int64, C.c_int,
                                           C.c_int, _i64p, _f32p, C.c_int]),
            "uvo_ivf_search_rerank": (None, [_vp, _f32p, C.c_int, _i64p, _i64p, _u8p, _u32p,
                                             _f32p, _f32p, C.c_int, _f32p, C.c_int64, C.c_int,
                                             C.c_int, C.c_int, _f32p, _i64p, _f32p, C.c_int]),
            "uvo_rand_unit": (None, [C.c_int64, C.c_int, C.c_uint64, _f32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Codec:
    """The reference TrellisQuantizer::from_config operating point
    (trellis.rs:352-458): seed 42, 3 rotation rounds, full free start."""

    def __init__(self, dim, bits, mem, seed=42, rounds=3, start_bits=None, rescale_bits=0,
                 branch_lambda=0.0, centroids=None):
        self.dim, self.bits, self.mem = dim, bits, mem
        sb = mem if start_bits is None else start_bits
        self.h = lib().uvo_codec_new(dim, bits, mem, seed, rounds, sb, rescale_bits,
                                     float(branch_lambda))
        if not self.h:
            raise ValueError("unsupported codec configuration")
        self.code_bytes = lib().uvo_codec_code_bytes(self.h)
        self.n_centroids = 0
        if centroids is not None:
            cen = np.ascontiguousarray(centroids, dtype=np.float32)
            lib().uvo_codec_set_centroids(self.h, cen, cen.shape[0])
            self.n_centroids = cen.shape[0]
        self.rounds = rounds

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().uvo_codec_free(self.h)
        except Exception:
            pass

    def table(self):
        out = np.empty(lib().uvo_codec_table_len(self.h), np.float32)
        lib().uvo_codec_table(self.h, out)
        return out

    def signs(self):
        out = np.empty(self.rounds * self.dim, np.float32)
        lib().uvo_codec_signs(self.h, out)
        return out.reshape(self.rounds, self.dim)

    def rotate(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        lib().uvo_rotate(self.h, x, out)
        return out

    def rotate_inverse(self, y):
        y = np.ascontiguousarray(y, np.float32)
        out = np.empty_like(y)
        lib().uvo_rotate_inverse(self.h, y, out)
        return out

    def encode(self, row):
        row = np.ascontiguousarray(row, np.float32)
        codes = np.zeros(self.code_bytes, np.uint8)
        st = np.zeros(1, np.uint32)
        rs = np.zeros(1, np.float32)
        rn = np.zeros(1, np.float32)
        ci = np.zeros(1, np.uint32)
        lib().uvo_encode(self.h, row, codes, st, rs, rn, ci)
        return codes, int(st[0]), float(rs[0]), float(rn[0]), int(ci[0])

    def encode_scalar_ref(self, row):
        row = np.ascontiguousarray(row, np.float32)
        codes = np.zeros(self.code_bytes, np.uint8)
        st = np.zeros(1, np.uint32)
        lib().uvo_encode_scalar_ref(self.h, row, codes, st)
        return codes, int(st[0])

    def encode_rotated(self, u_r):
        u_r = np.ascontiguousarray(u_r, np.float32)
        codes = np.zeros(self.code_bytes, np.uint8)
        st = np.zeros(1, np.uint32)
        lib().uvo_encode_rotated(self.h, u_r, codes, st)
        return codes, int(st[0])

    def encode_batch(self, rows, threads=0):
        rows = np.ascontiguousarray(rows, np.float32)
        n = rows.shape[0]
        codes = np.zeros((n, self.code_bytes), np.uint8)
        start = np.zeros(n, np.uint32)
        rescale = np.zeros(n, np.float32)
        rnorm = np.zeros(n, np.float32)
        cidx = np.zeros(n, np.uint32)
        lib().uvo_encode_batch(self.h, rows, n, codes, start, rescale, rnorm, cidx, threads)
        return dict(codes=codes, start=start, rescale=rescale, rnorm=rnorm, cidx=cidx)

    def encode_batch_signs(self, rows, threads=0):
        """encode_batch plus the shortlist sign codes (trellis.rs:1084-1094)."""
        rows = np.ascontiguousarray(rows, np.float32)
        n = rows.shape[0]
        out = dict(codes=np.zeros((n, self.code_bytes), np.uint8), start=np.zeros(n, np.uint32),
                   rescale=np.zeros(n, np.float32), rnorm=np.zeros(n, np.float32),
                   cidx=np.zeros(n, np.uint32),
                   signs=np.zeros((n, (self.dim + 7) // 8), np.uint8))
        lib().uvo_encode_batch_signs(self.h, rows, n, out["codes"], out["start"], out["rescale"],
                                     out["rnorm"], out["cidx"], out["signs"], threads)
        return out

    def ivf_encode_signs(self, rows, centroids, assign, threads=0):
        rows = np.ascontiguousarray(rows, np.float32)
        n = rows.shape[0]
        cen = None if centroids is None else np.ascontiguousarray(centroids, np.float32)
        out = dict(codes=np.zeros((n, self.code_bytes), np.uint8), start=np.zeros(n, np.uint32),
                   rescale=np.zeros(n, np.float32), rnorm=np.zeros(n, np.float32),
                   signs=np.zeros((n, (self.dim + 7) // 8), np.uint8))
        lib().uvo_ivf_encode_signs(self.h, rows, n, _ptr(cen),
                                   np.ascontiguousarray(assign, np.uint32), out["codes"],
                                   out["start"], out["rescale"], out["rnorm"], out["signs"],
                                   threads)
        return out

    def search_shortlist(self, index, queries, k, c, asym=False, weight=True, threads=0):
        """trellis.rs:854-948 for a flat index encoded with signs."""
        queries = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
        nq = queries.shape[0]
        ids = np.empty((nq, k), np.int64)
        scores = np.empty((nq, k), np.float32)
        rnorm = index.get("rnorm")
        cidx = index.get("cidx")
        lib().uvo_search_shortlist(
            self.h, np.ascontiguousarray(index["codes"], np.uint8),
            np.ascontiguousarray(index["start"], np.uint32),
            np.ascontiguousarray(index["rescale"], np.float32),
            _ptr(None if rnorm is None else np.ascontiguousarray(rnorm, np.float32)),
            _ptr(None if cidx is None else np.ascontiguousarray(cidx, np.uint32)),
            np.ascontiguousarray(index["signs"], np.uint8), index["start"].shape[0], queries, nq,
            k, c, int(asym), int(weight), ids, scores, threads)
        return ids, scores

    def ivf_search_shortlist(self, centroids, list_off, ids, index, centered, queries, nprobe,
                             k, c, asym=False, weight=True, threads=0):
        """ivf.rs:229-239 with TrellisShortlist{c, asym, rnorm=weight} lists."""
        queries = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
        nq = queries.shape[0]
        out_ids = np.empty((nq, k), np.int64)
        scores = np.empty((nq, k), np.float32)
        cen = np.ascontiguousarray(centroids, np.float32)
        lib().uvo_ivf_search_shortlist(
            self.h, cen, cen.shape[0], np.ascontiguousarray(list_off, np.int64),
            np.ascontiguousarray(ids, np.int64), np.ascontiguousarray(index["codes"], np.uint8),
            np.ascontiguousarray(index["start"], np.uint32),
            np.ascontiguousarray(index["rescale"], np.float32),
            np.ascontiguousarray(index["rnorm"], np.float32),
            np.ascontiguousarray(index["signs"], np.uint8), int(centered), queries, nq, nprobe,
            k, c, int(asym), int(weight), out_ids, scores, threads)
        return out_ids, scores

    def ivf_encode(self, rows, centroids, assign, threads=0):
        rows = np.ascontiguousarray(rows, np.float32)
        n = rows.shape[0]
        cen = None if centroids is None else np.ascontiguousarray(centroids, np.float32)
        assign = np.ascontiguousarray(assign, np.uint32)
        codes = np.zeros((n, self.code_bytes), np.uint8)
        start = np.zeros(n, np.uint32)
        rescale = np.zeros(n, np.float32)
        rnorm = np.zeros(n, np.float32)
        lib().uvo_ivf_encode(self.h, rows, n, _ptr(cen), assign, codes, start, rescale, rnorm,
                             threads)
        return dict(codes=codes, start=start, rescale=rescale, rnorm=rnorm)

    def windows(self, codes, start):
        out = np.empty(self.dim, np.uint32)
        lib().uvo_windows(self.h, np.ascontiguousarray(codes, np.uint8), start, out)
        return out

    def window_at(self, codes, start, i):
        return int(lib().uvo_window_at(self.h, np.ascontiguousarray(codes, np.uint8), start, i))

    def decode_codes(self, codes, start):
        out = np.empty(self.dim, np.float32)
        lib().uvo_decode_codes(self.h, np.ascontiguousarray(codes, np.uint8), start, out)
        return out

    def reconstruct_unit(self, codes, start, rnorm=1.0, cidx=0):
        out = np.empty(self.dim, np.float32)
        lib().uvo_reconstruct_unit(self.h, np.ascontiguousarray(codes, np.uint8), start,
                                   rnorm, cidx, out)
        return out

    def prepare_query(self, q):
        q = np.ascontiguousarray(q, np.float32)
        q_r = np.zeros(self.dim, np.float32)
        qc = np.zeros(max(1, self.n_centroids), np.float32)
        deg = lib().uvo_prepare_query(self.h, q, q_r, qc)
        return (None, None) if deg else (q_r, qc[: self.n_centroids])

    def search_topk(self, index, queries, k, norms=None, threads=0):
        queries = np.ascontiguousarray(queries, np.float32)
        nq = queries.shape[0]
        ids = np.empty((nq, k), np.int64)
        scores = np.empty((nq, k), np.float32)
        n = index["start"].shape[0]
        rnorm = index.get("rnorm")
        cidx = index.get("cidx")
        lib().uvo_search_topk(
            self.h, np.ascontiguousarray(index["codes"], np.uint8),
            np.ascontiguousarray(index["start"], np.uint32),
            np.ascontiguousarray(index["rescale"], np.float32),
            _ptr(None if rnorm is None else np.ascontiguousarray(rnorm, np.float32)),
            _ptr(None if cidx is None else np.ascontiguousarray(cidx, np.uint32)),
            _ptr(None if norms is None else np.ascontiguousarray(norms, np.float32)),
            n, queries, nq, k, ids, scores, threads)
        return ids, scores

    def score_candidates(self, index, queries, positions, offsets=None, threads=0):
        """trellis.rs:2016-2086: prepare each query, then score_at(positions[i])
        for the candidates offsets[q] <= i < offsets[q+1] (all on query 0
        without offsets)."""
        queries = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
        positions = np.ascontiguousarray(positions, np.int64)
        out = np.empty(positions.shape[0], np.float32)
        rnorm = index.get("rnorm")
        cidx = index.get("cidx")
        off = None if offsets is None else np.ascontiguousarray(offsets, np.int64)
        lib().uvo_score_candidates(
            self.h, np.ascontiguousarray(index["codes"], np.uint8),
            np.ascontiguousarray(index["start"], np.uint32),
            np.ascontiguousarray(index["rescale"], np.float32),
            _ptr(None if rnorm is None else np.ascontiguousarray(rnorm, np.float32)),
            _ptr(None if cidx is None else np.ascontiguousarray(cidx, np.uint32)),
            queries, queries.shape[0], _ptr(off), positions, positions.shape[0], out, threads)
        return out

    def ivf_search_topk(self, centroids, list_off, ids, index, centered, queries, nprobe, k,
                        threads=0):
        queries = np.ascontiguousarray(queries, np.float32)
        nq = queries.shape[0]
        out_ids = np.empty((nq, k), np.int64)
        scores = np.empty((nq, k), np.float32)
        cen = np.ascontiguousarray(centroids, np.float32)
        lib().uvo_ivf_search_topk(
            self.h, cen, cen.shape[0], np.ascontiguousarray(list_off, np.int64),
            np.ascontiguousarray(ids, np.int64), np.ascontiguousarray(index["codes"], np.uint8),
            np.ascontiguousarray(index["start"], np.uint32),
            np.ascontiguousarray(index["rescale"], np.float32),
            np.ascontiguousarray(index["rnorm"], np.float32), int(centered), queries, nq,
            nprobe, k, out_ids, scores, threads)
        return out_ids, scores

    def ivf_search_rerank(self, centroids, list_off, ids, index, centered, queries, nprobe, k,
                          rdepth, db, threads=0):
        """ivf.rs:248-274: codec top-max(rdepth, k), then exact cosine vs db."""
        queries = np.ascontiguousarray(queries, np.float32)
        nq = queries.shape[0]
        out_ids = np.empty((nq, k), np.int64)
        scores = np.empty((nq, k), np.float32)
        cen = np.ascontiguousarray(centroids, np.float32)
        lib().uvo_ivf_search_rerank(
            self.h, cen, cen.shape[0], np.ascontiguousarray(list_off, np.int64),
            np.ascontiguousarray(ids, np.int64), np.ascontiguousarray(index["codes"], np.uint8),
            np.ascontiguousarray(index["start"], np.uint32),
            np.ascontiguousarray(index["rescale"], np.float32),
            np.ascontiguousarray(index["rnorm"], np.float32), int(centered), queries, nq,
            nprobe, k, rdepth, np.ascontiguousarray(db, np.float32), out_ids, scores, threads)
        return out_ids, scores


def l2_norm(v):
    return float(lib().uvo_l2_norm(np.ascontiguousarray(v, np.float32), len(v)))


def l2_norms(rows, threads=0):
    """bench.rs:1019: exact l2 norm of every row (the MIPS sidecar)."""
    rows = np.ascontiguousarray(rows, np.float32)
    out = np.empty(rows.shape[0], np.float32)
    lib().uvo_l2_norms(rows, rows.shape[0], rows.shape[1], out, threads)
    return out


def std_about_mean(v):
    return float(lib().uvo_std_about_mean(np.ascontiguousarray(v, np.float32), len(v)))


def fwht(v):
    v = np.array(v, np.float32)
    lib().uvo_fwht(v, len(v))
    return v


def pack_indices(idx, bits):
    idx = np.ascontiguousarray(idx, np.uint16)
    out = np.zeros((len(idx) * bits + 7) // 8, np.uint8)
    lib().uvo_pack_indices(idx, len(idx), bits, out)
    return out


def unpack_indices(data, bits, n):
    out = np.zeros(n, np.uint16)
    data = np.ascontiguousarray(data, np.uint8)
    lib().uvo_unpack_indices(data, len(data), bits, out, n)
    return out


def lut_dot_u32(q, idx, book):
    return float(lib().uvo_lut_dot_u32(np.ascontiguousarray(q, np.float32),
                                       np.ascontiguousarray(idx, np.uint32),
                                       np.ascontiguousarray(book, np.float32), len(q)))


def dense_dot(a, b):
    return float(lib().uvo_dense_dot(np.ascontiguousarray(a, np.float32),
                                     np.ascontiguousarray(b, np.float32), len(a)))


def acs_step(cost, total, n_states, n_emit):
    nxt = np.zeros(n_states, np.float32)
    back = np.zeros(n_states, np.uint8)
    lib().uvo_acs_step(np.ascontiguousarray(cost, np.float32),
                       np.ascontiguousarray(total, np.float32), n_states, n_emit, nxt, back)
    return nxt, back


def digest(codes, start):
    codes = np.ascontiguousarray(codes, np.uint8)
    return int(lib().uvo_digest(codes, np.ascontiguousarray(start, np.uint32), codes.shape[0],
                                codes.shape[1]))


def exact_topk(db, queries, k, cosine=False, threads=0):
    db = np.ascontiguousarray(db, np.float32)
    queries = np.ascontiguousarray(queries, np.float32)
    ids = np.empty((queries.shape[0], k), np.int64)
    lib().uvo_exact_topk(db, db.shape[0], db.shape[1], queries, queries.shape[0], k,
                         int(cosine), ids, threads)
    return ids


def kmeans(db, nlist, seed=42, iters=5, threads=0):
    db = np.ascontiguousarray(db, np.float32)
    out = np.empty((nlist, db.shape[1]), np.float32)
    lib().uvo_kmeans(db, db.shape[0], db.shape[1], nlist, seed, iters, out, threads)
    return out


def assign(db, centroids, threads=0):
    db = np.ascontiguousarray(db, np.float32)
    cen = np.ascontiguousarray(centroids, np.float32)
    out = np.empty(db.shape[0], np.uint32)
    lib().uvo_assign(db, db.shape[0], db.shape[1], cen, cen.shape[0], out, threads)
    return out


def ivf_probe(centroids, query, nprobe):
    cen = np.ascontiguousarray(centroids, np.float32)
    out = np.empty(nprobe, np.int32)
    lib().uvo_ivf_probe(cen, cen.shape[0], cen.shape[1],
                        np.ascontiguousarray(query, np.float32), nprobe, out)
    return out


def rand_unit(n, dim, seed):
    out = np.empty((n, dim), np.float32)
    lib().uvo_rand_unit(n, dim, seed, out)
    return out


def threads_available() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


# ---------------------------------------------------------------------------
# Coset trellis (src/coset_trellis.rs, src/e8.rs)
# ---------------------------------------------------------------------------
def e8_key(r):
    return int(lib().uvo_e8_key(np.ascontiguousarray(r, np.int16)))


def e8_unkey(key):
    out = np.empty(8, np.int16)
    lib().uvo_e8_unkey(C.c_uint64(int(key)), out)
    return out


def coset_of(r):
    """coset_trellis.rs:73-79"""
    return int(lib().uvo_coset_of(np.ascontiguousarray(r, np.int16)))


def e8_nearest(y):
    """e8.rs:37-51"""
    out = np.empty(8, np.float32)
    lib().uvo_e8_nearest(np.ascontiguousarray(y, np.float32), out)
    return out


def e8_enumerate(r2_max):
    """e8.rs:82-92: every E8 point with |x|^2 <= r2_max, raw doubled coords."""
    n = lib().uvo_e8_enumerate(C.c_float(r2_max), None, 0)
    keys = np.empty(n, np.uint64)
    lib().uvo_e8_enumerate(C.c_float(r2_max), keys.ctypes.data, n)
    out = np.empty((n, 8), np.int16)
    for i, k in enumerate(keys):
        out[i] = e8_unkey(k)
    return out


class Coset:
    """CosetTrellis (coset_trellis.rs:98-190): dim % 8 == 0, bits 1..3, the
    reference defaults mem 12, rotation seed 42 and 3 rounds."""

    def __init__(self, dim, bits, mem=12, seed=42, rounds=3, centroids=None):
        self.dim, self.bits, self.mem = dim, bits, mem
        self.h = lib().uvo_coset_new(dim, bits, mem, seed, rounds)
        if not self.h:
            raise ValueError("unsupported coset trellis configuration")
        self.per_coset = lib().uvo_coset_per_coset(self.h)
        self.code_len = lib().uvo_coset_code_len(self.h)
        self.m_bits = 8 * bits - 3
        self.n_centroids = 0
        if centroids is not None:
            cen = np.ascontiguousarray(centroids, dtype=np.float32)
            lib().uvo_coset_set_centroids(self.h, cen, cen.shape[0])
            self.n_centroids = cen.shape[0]

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().uvo_coset_free(self.h)
        except Exception:
            pass

    def books(self):
        """8 x per_coset keys (norm << 40 | offset coordinates)."""
        out = np.empty(8 * self.per_coset, np.uint64)
        lib().uvo_coset_books(self.h, out)
        return out.reshape(8, self.per_coset)

    def book_points(self, k):
        keys = self.books()[k]
        sh = np.array([35, 30, 25, 20, 15, 10, 5, 0], np.uint64)
        return (((keys[:, None] >> sh[None, :]) & np.uint64(31)).astype(np.int16) - 16)

    def scale(self):
        out = np.empty(2, np.float32)
        lib().uvo_coset_scale(self.h, out)
        return float(out[0]), float(out[1])

    def index(self, k, r):
        return int(lib().uvo_coset_index(self.h, k, np.ascontiguousarray(r, np.int16)))

    def nearest(self, k, y, exhaustive=False):
        i, d = C.c_int64(), C.c_float()
        fn = lib().uvo_coset_nearest_exhaustive if exhaustive else lib().uvo_coset_nearest
        fn(self.h, k, np.ascontiguousarray(y, np.float32), C.byref(i), C.byref(d))
        return i.value, d.value

    def encode_batch(self, rows):
        rows = np.ascontiguousarray(rows, np.float32)
        n = rows.shape[0]
        codes = np.zeros((n, self.code_len), np.uint8)
        rescale = np.empty(n, np.float32)
        rnorm = np.empty(n, np.float32)
        cidx = np.empty(n, np.uint32)
        lib().uvo_coset_encode_batch(self.h, rows, n, codes, rescale, rnorm, cidx)
        return {"codes": codes, "rescale": rescale, "rnorm": rnorm, "cidx": cidx}

    def decode(self, rec):
        out = np.empty(self.dim, np.float32)
        lib().uvo_coset_decode(self.h, np.ascontiguousarray(rec, np.uint8), out)
        return out

    def reconstruct_unit(self, row):
        out = np.empty(self.dim, np.float32)
        lib().uvo_coset_reconstruct_unit(self.h, np.ascontiguousarray(row, np.float32), out)
        return out

    def search(self, enc, queries, k, ids=None):
        queries = np.ascontiguousarray(queries, np.float32)
        nq = queries.shape[0]
        n = enc["codes"].shape[0]
        out_ids = np.empty((nq, k), np.int64)
        out_sc = np.empty((nq, k), np.float32)
        ids_arr = None if ids is None else np.ascontiguousarray(ids, np.int64)
        lib().uvo_coset_search(self.h, np.ascontiguousarray(enc["codes"]), enc["rescale"],
                               enc["rnorm"], enc["cidx"],
                               None if ids_arr is None else ids_arr.ctypes.data, n, queries,
                               nq, k, out_ids, out_sc)
        return out_ids, out_sc

    def mem_bytes(self, n):
        return int(lib().uvo_coset_mem_bytes(self.h, n))

