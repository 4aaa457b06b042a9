"""ctypes binding of ``libbgattn.so`` (the C ABI declared in ``include/bgattn.h``).

The library is required: importing this module on a machine without the built ``.so`` raises,
and there is no CPU fallback anywhere in the package.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("BGATTN_LIB") or os.path.join(HERE, "libbgattn.so")  # override: A/B builds

BG_OK, BG_EINVAL, BG_ENOMEM, BG_ELAUNCH, BG_ETIMEOUT, BG_EUNSUPPORTED = 0, -1, -2, -3, -4, -5
KV_F32, KV_F16, KV_Q8, KV_Q8R = 0, 1, 2, 3
DT_F32, DT_F16 = 0, 1

# every symbol include/bgattn.h declares (checked by the CPU test suite)
EXPORTS = [
    "bg_strerror", "bg_version", "bg_device_status", "bg_force_generic", "bg_attention_workspace_size", "bg_attention", "bg_attention_partials",
    "bg_lse_merge", "bg_kv_append", "bg_kv_append_kv", "bg_rmsnorm_rope", "bg_kv_evict", "bg_kv_ring_evict",
    "bg_deltanet_gbeta", "bg_deltanet_recur", "bg_deltanet_norm_gate", "bg_deltanet_fused",
    "bg_gate_sigmoid", "bg_attention_noalloc", "bg_deltanet_chunked_workspace_size",
    "bg_deltanet_chunked", "bg_qk_norm_rope", "bg_conv1d_causal", "bg_slice_cols",
    "bg_kv_snapshot_bytes", "bg_kv_snapshot_save", "bg_kv_snapshot_restore", "bg_attention_noalloc_limit",
    "bg_selftest_wait_expiry", "bg_kv_append_kv_pair", "bg_peer_exchange_bytes", "bg_peer_exchange_flags_offset",
    "bg_attention_peer_workspace_size", "bg_attention_peer",
]


class AttnParams(C.Structure):
    _fields_ = [("S", C.c_uint32), ("H", C.c_uint32), ("KV", C.c_uint32), ("D", C.c_uint32),
                ("posBase", C.c_uint32), ("Ltot", C.c_uint32)]


class KVCacheDesc(C.Structure):
    _fields_ = [("K", C.c_void_p), ("V", C.c_void_p), ("Ks", C.c_void_p), ("Vs", C.c_void_p),
                ("seq_stride", C.c_uint64), ("mode", C.c_uint32), ("sinks", C.c_uint32),
                ("window", C.c_uint32), ("ring_head", C.c_uint32)]


MAX_PEERS = 8


class PeerExchange(C.Structure):
    _fields_ = [("nranks", C.c_uint32), ("rank", C.c_uint32), ("gather", C.c_void_p * MAX_PEERS),
                ("flags", C.c_void_p * MAX_PEERS), ("step", C.c_void_p), ("done", C.c_void_p),
                ("tickets", C.c_void_p), ("spin_limit", C.c_uint32)]


class BgError(RuntimeError):
    def __init__(self, fn, code):
        super().__init__(f"{fn} failed: {code} ({lib().bg_strerror(code).decode()})")
        self.code = code


_LIB = None

P, U32, U64, F, SZ = C.c_void_p, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t
_SIGS = {
    "bg_strerror": (C.c_char_p, [C.c_int]),
    "bg_version": (C.c_int, []),
    "bg_device_status": (C.c_int, [P]),
    "bg_force_generic": (C.c_int, [C.c_int]),
    "bg_attention_workspace_size": (SZ, [C.POINTER(AttnParams), U32]),
    "bg_attention": (C.c_int, [C.POINTER(AttnParams), U32, P, U32, C.POINTER(KVCacheDesc), P, P, F, P, P, U32, P,
                               SZ, P]),
    "bg_attention_partials": (C.c_int, [C.POINTER(AttnParams), U32, P, U32, C.POINTER(KVCacheDesc), P, P, F, U32,
                                        U32, P, P, SZ, P]),
    "bg_lse_merge": (C.c_int, [P, U32, U32, U32, P, P, U32, P]),
    "bg_kv_append": (C.c_int, [C.POINTER(KVCacheDesc), U32, U32, P, U32, U32, U32, U32, U32, P]),
    "bg_kv_append_kv": (C.c_int, [C.POINTER(KVCacheDesc), U32, P, P, U32, U32, U32, U32, U32, P]),
    "bg_kv_append_kv_pair": (C.c_int, [C.POINTER(KVCacheDesc), C.POINTER(KVCacheDesc), U32, P, P, U32, U32, U32, U32,
                                       U32, P]),
    "bg_qk_norm_rope": (C.c_int, [P, U32, U32, U32, U32, U32, U32, P, P, P, U32, U32, F, P,
                                  C.POINTER(KVCacheDesc), P]),
    "bg_conv1d_causal": (C.c_int, [P, P, P, U32, U32, U32, U32, P, P, P]),
    "bg_slice_cols": (C.c_int, [P, U32, U32, U32, U32, P, P]),
    "bg_kv_snapshot_bytes": (SZ, [C.POINTER(KVCacheDesc), U32, U32, U32]),
    "bg_kv_snapshot_save": (C.c_int, [C.POINTER(KVCacheDesc), U32, U32, U32, U32, U32, P, P]),
    "bg_kv_snapshot_restore": (C.c_int, [C.POINTER(KVCacheDesc), U32, U32, U32, U32, U32, P, P]),
    "bg_rmsnorm_rope": (C.c_int, [P, U32, U32, U32, P, P, P, F, P, C.POINTER(KVCacheDesc), U32, P]),
    "bg_kv_evict": (C.c_int, [C.POINTER(KVCacheDesc), U32, U32, U32, U32, U32, U32, C.POINTER(U32), P]),
    "bg_kv_ring_evict": (C.c_int, [C.POINTER(KVCacheDesc), U32, U32, U32, C.POINTER(U32)]),
    "bg_deltanet_gbeta": (C.c_int, [P, P, P, P, U32, U32, P, P]),
    "bg_deltanet_recur": (C.c_int, [C.POINTER(U32 * 8), P, P, P, P, P, P, P, P, P]),
    "bg_deltanet_norm_gate": (C.c_int, [P, P, P, U32, U32, F, P, P]),
    "bg_deltanet_fused": (C.c_int, [U32, U32, U32, U32, U32, P, P, P, P, P, P, P, P, P, F, P, P, P, P, P]),
    "bg_gate_sigmoid": (C.c_int, [P, P, U32, P, P]),
    "bg_deltanet_chunked_workspace_size": (SZ, [U32, U32, U32, U32]),
    "bg_deltanet_chunked": (C.c_int, [U32, U32, U32, U32, U32, P, P, P, P, P, P, P, P, P, F, P, P, P, P, P, SZ, P]),
    "bg_attention_noalloc_limit": (SZ, []),
    "bg_peer_exchange_bytes": (SZ, [U32, U32, U32]),
    "bg_peer_exchange_flags_offset": (SZ, [U32, U32, U32]),
    "bg_attention_peer_workspace_size": (SZ, [C.POINTER(AttnParams), U32]),
    "bg_attention_peer": (C.c_int, [C.POINTER(AttnParams), U32, P, U32, C.POINTER(KVCacheDesc), F, U32, U32,
                                    C.POINTER(PeerExchange), P, P, U32, P, SZ, P]),
    "bg_selftest_wait_expiry": (C.c_int, [U32, P]),
    "bg_attention_noalloc": (C.c_int, [C.POINTER(AttnParams), U32, P, U32, C.POINTER(KVCacheDesc), P, P, F, P, P,
                                       U32, P]),
}


def lib():
    """Load (once) and return the library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m bitgpu_b200.build` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(fn, code):
    if code != BG_OK:
        raise BgError(fn, code)
