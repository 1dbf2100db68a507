"""ultravec-ann_b200: B200-native (sm_100a) trellis encoder and codes-only
scan behind a C ABI (include/ultravec_b200.h).

The directory name is not a Python identifier, so the package is registered
as `ultravec_ann_b200` by `load()` in ultravec_ann_b200_loader.py (repo root)
or by any importer that points importlib at this directory.
"""
from .binding import (Codec, CosetIndex, Index, IvfIndex, PreparedQueries, ShardSearch,  # noqa: F401
                      UVError, build, check, ivf_assign, kmeans, lib, topk_merge,
                      topk_merge_packed, topk_pack, topk_unpack, profile_enable, profile_read,
                      set_tuning, UV_SEARCH_COSINE, UV_SEARCH_MIPS, SYMBOLS)
