"""ctypes bindings of the oracle libraries -- test infrastructure only.

  _build/libgdn_oracle.so   the C restatement (gdn_oracle.c)
  _build/libgdn_cpu_port.so CPU decode step over the restatement's codec
  _ref/libgdn_ref.so        the reference's own quantiser / dequantiser /
                            GPU op path, compiled from its sources (may be absent)
  _ref/libgdn_cpu_ref.so    CPU decode step over the reference's host codec

Numpy in, numpy out.  bf16 arrays travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF = HERE / "_ref"

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_f64 = ctypes.c_double
_u32 = ctypes.c_uint32


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def _load(path: pathlib.Path, sigs: dict) -> ctypes.CDLL:
    if not path.exists():
        raise FileNotFoundError(f"{path} missing: run `make -C oracle` (and `make -C oracle ref`)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_ORACLE_SIGS = {
    "orc_e2m1_decode": (_f32, [_u32]),
    "orc_e2m1_encode": (_u32, [_f32]),
    "orc_scale_decode": (_f32, [_u32, ctypes.c_int]),
    "orc_scale_encode": (_u32, [_f32, ctypes.c_int]),
    "orc_quantise": (None, [_p, _p, _p, _i64, ctypes.c_int]),
    "orc_dequantise": (None, [_p, _p, _p, _i64, ctypes.c_int]),
    "orc_global_scale": (_f32, [_p, _i64, _f32]),
    "orc_quantise_tile_gs": (None, [_p, _i64, _p, _p, _p, _p, ctypes.c_int, _f32]),
    "orc_dequantise_tile_gs": (None, [_p, _p, _f32, _p, _i64, ctypes.c_int]),
    "orc_legacy_update_f32": (None, [_p, _p, _p, _p, _f32, _f32, ctypes.c_int, ctypes.c_int]),
    "orc_legacy_op": (None, [_p, _p, _p, _p, _p, _p, _f32, _f32, ctypes.c_int, ctypes.c_int]),
    "orc_gdn_decode": (None, [ctypes.c_int] * 4 + [_p] * 11 + [_f32, ctypes.c_int, _f32, _p]),
    "orc_gdn_recurrent_f64": (None, [ctypes.c_int, ctypes.c_int, _p, _p, _p, _p, _i64, _i64, _p, _p, _i64, _p,
                                     _i64, _f64]),
    "orc_gdn_chunked_f64": (None, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p, _p, _p, _i64, _i64, _p, _p,
                                   _i64, _p, _i64, _f64]),
    "orc_sqnr_db": (_f64, [_p, _p, _i64]),
    "orc_scale_encode_sweep": (None, [_u32, _u32, ctypes.c_uint64, ctypes.c_int, _p]),
    "orc_block_scale_sweep": (None, [_u32, ctypes.c_uint64, ctypes.c_int, _p]),
    "orc_e2m1_sweep": (None, [_u32, ctypes.c_uint64, _p]),
    "orc_libc_srand": (None, [ctypes.c_uint]),
    "orc_libc_fill_uniform": (None, [_p, _i64, _f32, _f32]),
}

_REF_SIGS = {
    "ref_nvfp4_quantise": (None, [_p, _p, _p, ctypes.c_int]),
    "ref_nvfp4_dequantise": (None, [_p, _p, _p, ctypes.c_int]),
    "ref_decode_e2m1": (_f32, [_u32]),
    "ref_decode_ue4m3": (_f32, [_u32]),
    "ref_encode_ue4m3": (_u32, [_f32]),
    "ref_encode_ue4m3_sweep": (None, [_u32, _u32, ctypes.c_uint64, _p]),
    "ref_block_scale_sweep": (None, [_u32, ctypes.c_uint64, _p]),
    "ref_e2m1_sweep": (None, [_u32, ctypes.c_uint64, _p]),
    "launch_gdn_state_update": (ctypes.c_int, [_p, _p, _p, _p, _p, _p, _f32, _f32, ctypes.c_int, _p]),
    "launch_gdn_ref": (None, [_p, _p, _p, _p, _p, _f32, _f32, ctypes.c_int, _p]),
}

_CPU_SIGS = {
    "cpu_gdn_decode": (_i64, [ctypes.c_int] * 4 + [_p] * 10 + [_f32, ctypes.c_int, _f32, _i64, _i64,
                                                                  ctypes.c_int]),
    "cpu_max_threads": (ctypes.c_int, []),
    "cpu_baseline_uses_reference": (ctypes.c_int, []),
}

_oracle = None
_ref = None


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        _oracle = _load(BUILD / "libgdn_oracle.so", _ORACLE_SIGS)
    return _oracle


def ref_available() -> bool:
    return (REF / "libgdn_ref.so").exists()


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        _ref = _load(REF / "libgdn_ref.so", _REF_SIGS)
    return _ref


def cpu_baseline(prefer_reference: bool = True) -> tuple[ctypes.CDLL, str]:
    """(library, kind) for the timed CPU decode step: the reference-codec build
    when present ("reference"), else the restatement ("port")."""
    if prefer_reference and (REF / "libgdn_cpu_ref.so").exists():
        return _load(REF / "libgdn_cpu_ref.so", _CPU_SIGS), "reference"
    return _load(BUILD / "libgdn_cpu_port.so", _CPU_SIGS), "port"


# ---- numpy wrappers ------------------------------------------------------------

def quantise(x: np.ndarray, mode: int = 0) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    codes = np.zeros(x.size // 2, np.uint8)
    scales = np.zeros(x.size // 16, np.uint8)
    oracle().orc_quantise(_ptr(x), _ptr(codes), _ptr(scales), x.size, mode)
    return codes, scales


def dequantise(codes: np.ndarray, scales: np.ndarray, mode: int = 0) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1)
    scales = np.ascontiguousarray(scales, np.uint8).reshape(-1)
    out = np.zeros(codes.size * 2, np.float32)
    oracle().orc_dequantise(_ptr(codes), _ptr(scales), _ptr(out), out.size, mode)
    return out


def quantise_tiles(x: np.ndarray, tile_elems: int, mode: int = 0, gden: float = 0.0):
    """Per-tile global scale + reference quantiser: (codes, scales, gscale, y)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if gden <= 0:
        gden = 6.0 * (448.0 if mode else 240.0)
    nt = x.size // tile_elems
    codes = np.zeros(x.size // 2, np.uint8)
    scales = np.zeros(x.size // 16, np.uint8)
    gs = np.zeros(nt, np.float32)
    y = np.zeros(x.size, np.float32)
    for t in range(nt):
        sl = slice(t * tile_elems, (t + 1) * tile_elems)
        g = np.zeros(1, np.float32)
        xt = np.ascontiguousarray(x[sl])
        ct = np.zeros(tile_elems // 2, np.uint8)
        st = np.zeros(tile_elems // 16, np.uint8)
        yt = np.zeros(tile_elems, np.float32)
        oracle().orc_quantise_tile_gs(_ptr(xt), tile_elems, _ptr(ct), _ptr(st), _ptr(g), _ptr(yt), mode, gden)
        codes[t * tile_elems // 2:(t + 1) * tile_elems // 2] = ct
        scales[t * tile_elems // 16:(t + 1) * tile_elems // 16] = st
        gs[t] = g[0]
        y[sl] = yt
    return codes, scales, gs, y


def dequantise_tiles(codes: np.ndarray, scales: np.ndarray, gs: np.ndarray, mode: int = 0) -> np.ndarray:
    out = dequantise(codes, scales, mode)
    nt = gs.size
    return (out.reshape(nt, -1) * gs.reshape(nt, 1).astype(np.float32)).reshape(-1)


def ref_quantise(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The reference's own nvfp4_quantise_host (mode 0)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    codes = np.zeros(x.size // 2, np.uint8)
    scales = np.zeros(x.size // 16, np.uint8)
    ref().ref_nvfp4_quantise(_ptr(x), _ptr(codes), _ptr(scales), x.size)
    return codes, scales


def ref_dequantise(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1)
    scales = np.ascontiguousarray(scales, np.uint8).reshape(-1)
    out = np.zeros(codes.size * 2, np.float32)
    ref().ref_nvfp4_dequantise(_ptr(codes), _ptr(scales), _ptr(out), out.size)
    return out


def legacy_update_f32(S: np.ndarray, k_bf16: np.ndarray, v_bf16: np.ndarray, alpha: float, beta: float,
                      variant: int) -> np.ndarray:
    d = k_bf16.size
    S = np.ascontiguousarray(S, np.float32).reshape(-1)
    out = np.zeros(d * d, np.float32)
    oracle().orc_legacy_update_f32(_ptr(S), _ptr(np.ascontiguousarray(k_bf16, np.uint16)),
                                   _ptr(np.ascontiguousarray(v_bf16, np.uint16)), _ptr(out), alpha, beta, d,
                                   variant)
    return out


def legacy_op(S_data, S_scales, k_bf16, v_bf16, alpha: float, beta: float, d: int, variant: int):
    out_d = np.zeros(d * d // 2, np.uint8)
    out_s = np.zeros(d * d // 16, np.uint8)
    oracle().orc_legacy_op(_ptr(np.ascontiguousarray(S_data, np.uint8)), _ptr(np.ascontiguousarray(S_scales, np.uint8)),
                           _ptr(np.ascontiguousarray(k_bf16, np.uint16)), _ptr(np.ascontiguousarray(v_bf16, np.uint16)),
                           _ptr(out_d), _ptr(out_s), alpha, beta, d, variant)
    return out_d, out_s


def gdn_decode(q, k, v, g, beta, slot, codes, scales, gs, q_scale: float, mode: int = 0, gden: float = 0.0,
               want_y: bool = False):
    """One decode step of the oracle.  q, k: [B, HK, D] uint16 (bf16 bits);
    v: [B, HV, D] uint16; g, beta: [B, HV] f32; slot: [B] int32; codes, scales,
    gs: the pool (updated in place, must be C-contiguous numpy arrays).
    Returns (o_f32 [B, HV, D], o_bf16 bits, y or None)."""
    B, HK, D = q.shape
    HV = v.shape[1]
    if gden <= 0:
        gden = 6.0 * (448.0 if mode else 240.0)
    o32 = np.zeros((B, HV, D), np.float32)
    o16 = np.zeros((B, HV, D), np.uint16)
    y = np.zeros((B, HV, D, D), np.float32) if want_y else None
    arrs = [np.ascontiguousarray(a) for a in (q, k, v, g, beta, slot)]
    for a in (codes, scales, gs):
        assert a.flags["C_CONTIGUOUS"]
    oracle().orc_gdn_decode(B, HK, HV, D, *[_ptr(a) for a in arrs], _ptr(codes), _ptr(scales), _ptr(gs),
                            _ptr(o16), _ptr(o32), q_scale, mode, gden, _ptr(y))
    return o32, o16, y


def recurrent_f64(S0: np.ndarray, q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray, beta: np.ndarray,
                  q_scale: float):
    """Unquantised recurrence of one (sequence, head): S0 [D, D] f64 (copied),
    q, k, v [T, D] f32, g, beta [T] f32.  Returns (o [T, D] f64, S_T [D, D])."""
    T, D = q.shape
    S = np.array(S0, dtype=np.float64, order="C", copy=True)
    o = np.zeros((T, D), np.float64)
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    g, beta = (np.ascontiguousarray(a, np.float32) for a in (g, beta))
    oracle().orc_gdn_recurrent_f64(T, D, _ptr(S), _ptr(q), _ptr(k), _ptr(v), D, D, _ptr(g), _ptr(beta), 1, _ptr(o),
                                   D, q_scale)
    return o, S


def chunked_f64(S0: np.ndarray, q, k, v, g, beta, q_scale: float, chunk: int = 64):
    T, D = q.shape
    S = np.array(S0, dtype=np.float64, order="C", copy=True)
    o = np.zeros((T, D), np.float64)
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    g, beta = (np.ascontiguousarray(a, np.float32) for a in (g, beta))
    oracle().orc_gdn_chunked_f64(T, D, chunk, _ptr(S), _ptr(q), _ptr(k), _ptr(v), D, D, _ptr(g), _ptr(beta), 1,
                                 _ptr(o), D, q_scale)
    return o, S


def sqnr_db(ref_arr: np.ndarray, test_arr: np.ndarray) -> float:
    a = np.ascontiguousarray(ref_arr, np.float64).reshape(-1)
    b = np.ascontiguousarray(test_arr, np.float64).reshape(-1)
    return float(oracle().orc_sqnr_db(_ptr(a), _ptr(b), a.size))


def m3_fixture(d_list=(512, 1024, 2048), seed: int = 42):
    """The reference M3 gate's inputs (tests/test_gdn_correctness.cu:200,
    :101-104, :216-218): after srand(42), for each d in turn, S ~ U(-4, 4)
    [d*d], k, v ~ U(-1, 1) [d], drawn from the C library's rand() in float.
    Yields (d, S, k, v) as float32 arrays."""
    oracle().orc_libc_srand(seed)
    for d in d_list:
        S = np.zeros(d * d, np.float32)
        k = np.zeros(d, np.float32)
        v = np.zeros(d, np.float32)
        oracle().orc_libc_fill_uniform(_ptr(S), S.size, -4.0, 4.0)
        oracle().orc_libc_fill_uniform(_ptr(k), k.size, -1.0, 1.0)
        oracle().orc_libc_fill_uniform(_ptr(v), v.size, -1.0, 1.0)
        yield d, S, k, v


def scale_encode_sweep(lo: int, stride: int, count: int, mode: int = 0) -> np.ndarray:
    out = np.zeros(count, np.uint8)
    oracle().orc_scale_encode_sweep(lo, stride, count, mode, _ptr(out))
    return out


def ref_scale_encode_sweep(lo: int, stride: int, count: int) -> np.ndarray:
    out = np.zeros(count, np.uint8)
    ref().ref_encode_ue4m3_sweep(lo, stride, count, _ptr(out))
    return out


def _threaded_sweep(fn, lo: int, count: int, threads: int | None, *extra) -> np.ndarray:
    """Runs fn(lo_i, count_i, *extra, out_i) on `threads` slices of the range
    in parallel (ctypes releases the GIL during the call)."""
    import concurrent.futures
    import os
    out = np.zeros(count, np.uint8)
    threads = threads or max(1, len(os.sched_getaffinity(0)))
    step = -(-count // threads)
    step += (-step) % 15  # keep the reference's 15-value groups whole
    jobs = []
    with concurrent.futures.ThreadPoolExecutor(threads) as ex:
        for s0 in range(0, count, step):
            n = min(step, count - s0)
            view = out[s0:s0 + n]
            jobs.append(ex.submit(fn, lo + s0, n, *extra, view.ctypes.data))
        for j in jobs:
            j.result()
    return out


def block_scale_sweep(lo: int, count: int, mode: int = 0, threads: int | None = None) -> np.ndarray:
    """Oracle block scale byte of every block max with bit pattern lo + i."""
    return _threaded_sweep(lambda a, n, m, o: oracle().orc_block_scale_sweep(a, n, m, o), lo, count, threads, mode)


def e2m1_sweep(lo: int, count: int, threads: int | None = None) -> np.ndarray:
    """Oracle E2M1 nibble of every value with bit pattern lo + i."""
    return _threaded_sweep(lambda a, n, o: oracle().orc_e2m1_sweep(a, n, o), lo, count, threads)


def ref_block_scale_sweep(lo: int, count: int, threads: int | None = None) -> np.ndarray:
    """The reference's block scale byte (amax/6 through its encoder), bit patterns lo + i."""
    return _threaded_sweep(lambda a, n, o: ref().ref_block_scale_sweep(a, n, o), lo, count, threads)


def ref_e2m1_sweep(lo: int, count: int, threads: int | None = None) -> np.ndarray:
    """The reference quantiser's E2M1 nibble of every value (|v| <= 6) with bit pattern lo + i."""
    return _threaded_sweep(lambda a, n, o: ref().ref_e2m1_sweep(a, n, o), lo, count, threads)


# ---- helpers shared by tests and the bench ----------------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)
