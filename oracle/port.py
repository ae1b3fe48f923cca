"""ctypes wrapper of oracle/_build/liboc_port.so — the CPU port of the
reference's decode step (see oc_port.c).  Test / baseline infrastructure."""
import ctypes as C
import os

import numpy as np

from .build_port import OUT, build

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(OUT):
            build()
        _lib = C.CDLL(OUT)
        _lib.oc_port_decode.restype = C.c_int
        _lib.oc_port_threads.restype = C.c_int
    return _lib


def threads():
    return lib().oc_port_threads()


def scores(k_bits, q_bits):
    """(bound_max, zeta) float32 (nb, Hkv) of the two gates, from the port."""
    S, H, D = k_bits.shape
    Sq, Hq, _ = q_bits.shape
    nb = S // 512
    bmax = np.zeros((nb, H), np.float32)
    zeta = np.zeros((nb, H), np.float32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    lib().oc_port_scores(p(k_bits), p(q_bits), S, H, Hq, D, Sq, p(bmax), p(zeta))
    return bmax, zeta


def decode(k_bits, v_bits, q_bits, tau, zeta_max, blocks_limit=0):
    """k_bits/v_bits (S,Hkv,D), q_bits (Sq,Hq,D): uint16 bf16 bit patterns.
    Returns keep (nb,Hkv) bool, perm (nb,), count, out (Sq,Hq,D) f32."""
    S, H, D = k_bits.shape
    Sq, Hq, _ = q_bits.shape
    nb = S // 512
    keep = np.zeros((nb, H), np.uint8)
    perm = np.zeros(nb, np.int32)
    count = np.zeros(1, np.int32)
    out = np.zeros((Sq, Hq, D), np.float32)
    ck = np.empty_like(k_bits)
    cv = np.empty_like(v_bits)
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    lib().oc_port_decode(p(k_bits), p(v_bits), p(q_bits), S, H, Hq, D, Sq, C.c_float(tau),
                         C.c_float(zeta_max), blocks_limit, p(keep), p(perm), p(count), p(out), p(ck), p(cv))
    return keep.astype(bool), perm, int(count[0]), out
