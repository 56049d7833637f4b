"""ctypes binding of ``libt2w_b200.so`` (the C ABI declared in ``include/t2w_b200.h``).

There is no fallback: if the library is missing or the device is not an sm_100 GPU, calls raise.  Status codes become
``T2WError`` exceptions carrying the C status and, for CUDA failures, the CUDA error code.
"""

from __future__ import annotations

import ctypes
import os
import re

from .build import INCLUDE, LIB_PATH

T2W_OK = 0
STATUS = {-1: "invalid argument or shape", -2: "CUDA error", -3: "out of device memory", -4: "kernel wait timed out",
          -5: "unsupported config or device", -6: "workspace too small",
          -7: "Token2Wav cache pool exhausted (key slots, conv-cache row slots or cache handles)"}
PREC = {"bf16": 0, "fp8": 1}
FLAG_GRAPH = 1
EPI = {"f32": 0, "bf16": 1, "gelu": 2, "resid": 3, "qkv": 4, "silu": 5, "leaky": 6, "gelu_fp8": 8}
KERNEL_CLASSES = ["pack", "gemm_in", "ln_mod", "gemm_qkv", "attn", "gemm_proj", "gemm_conv1", "ln_mish", "gemm_conv2",
                  "gemm_fc1", "gemm_fc2", "gemm_final", "euler"]
W_GLOBAL = ["estimator.t_embedder.mlp.0.weight", "estimator.t_embedder.mlp.0.bias", "estimator.t_embedder.mlp.2.weight",
            "estimator.t_embedder.mlp.2.bias", "estimator.in_proj.weight", "estimator.in_proj.bias",
            "estimator.final_layer.adaLN_modulation.1.weight", "estimator.final_layer.adaLN_modulation.1.bias",
            "estimator.final_layer.linear.weight", "estimator.final_layer.linear.bias"]
W_BLOCK = ["adaLN_modulation.1.weight", "adaLN_modulation.1.bias", "attn.to_q.weight", "attn.to_q.bias",
           "attn.to_k.weight", "attn.to_k.bias", "attn.to_v.weight", "attn.to_v.bias", "attn.q_norm.weight",
           "attn.q_norm.bias", "attn.k_norm.weight", "attn.k_norm.bias", "attn.proj.weight", "attn.proj.bias",
           "conv.block.1.weight", "conv.block.1.bias", "conv.block.3.weight", "conv.block.3.bias", "conv.block.6.weight",
           "conv.block.6.bias", "mlp.fc1.weight", "mlp.fc1.bias", "mlp.fc2.weight", "mlp.fc2.bias"]


class T2WError(RuntimeError):
    def __init__(self, fn: str, status: int, cuda: int = 0):
        msg = f"{fn} failed: {STATUS.get(status, 'unknown')} (status {status}"
        msg += f", cudaError {cuda})" if status == -2 else ")"
        super().__init__(msg)
        self.status, self.cuda = status, cuda


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("mel", "hidden", "depth", "heads", "head_dim", "ffn", "steps", "freq_dim")] + \
               [(n, ctypes.c_float) for n in ("cfg_rate", "t_scale", "max_period", "eps_block", "eps_final", "eps_qk", "eps_conv")]


class Batch(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_int32), ("prompt_len", ctypes.POINTER(ctypes.c_int32)),
                ("chunk_len", ctypes.POINTER(ctypes.c_int32)), ("x0", ctypes.c_void_p), ("mu", ctypes.c_void_p),
                ("cond", ctypes.c_void_p), ("spk", ctypes.c_void_p), ("out", ctypes.c_void_p)]


class SlotBatch(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_int32)] + \
               [(n, ctypes.POINTER(ctypes.c_int32)) for n in ("chunk_len", "kv_len", "kv_idx", "cnn_rd", "cnn_wr")] + \
               [(n, ctypes.c_void_p) for n in ("x0", "mu", "cond", "spk", "out")]


class CacheInfo(ctypes.Structure):
    _fields_ = [("length", ctypes.c_int32), ("keep", ctypes.c_int32), ("rowslot", ctypes.c_int32 * 2)]


class CachedBatch(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_int32), ("handle", ctypes.POINTER(ctypes.c_int32)),
                ("chunk_len", ctypes.POINTER(ctypes.c_int32)), ("keep", ctypes.POINTER(ctypes.c_uint8)),
                ("noise", ctypes.c_void_p), ("noise_frames", ctypes.c_int32), ("temperature", ctypes.c_float),
                ("mu", ctypes.c_void_p), ("cond", ctypes.c_void_p), ("spk", ctypes.c_void_p), ("out", ctypes.c_void_p)]


class EncConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("vocab", "hidden", "heads", "head_dim", "ffn", "blocks1", "blocks2",
                                              "stride", "lookahead", "mel")] + \
               [(n, ctypes.c_float) for n in ("eps_layer", "eps_embed", "eps_after", "leaky_slope", "max_period")]


class EncBatch(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_int32), ("handle", ctypes.POINTER(ctypes.c_int32)),
                ("n_tokens", ctypes.POINTER(ctypes.c_int32)), ("final", ctypes.POINTER(ctypes.c_uint8)),
                ("tokens", ctypes.POINTER(ctypes.c_int32)), ("mu", ctypes.c_void_p)]


# Flow-encoder weight slots (include/t2w_b200.h t2w_enc_weight_slot / t2w_enc_layer_slot): state-dict paths of the flow
# module (input_embedding, encoder.*, encoder_proj).
E_GLOBAL = ["input_embedding.weight", "encoder.embed.out.0.weight", "encoder.embed.out.0.bias",
            "encoder.embed.out.1.weight", "encoder.embed.out.1.bias", "encoder.pre_lookahead_layer.conv1.weight",
            "encoder.pre_lookahead_layer.conv1.bias", "encoder.pre_lookahead_layer.conv2.weight",
            "encoder.pre_lookahead_layer.conv2.bias", "encoder.up_layer.conv.weight", "encoder.up_layer.conv.bias",
            "encoder.up_embed.out.0.weight", "encoder.up_embed.out.0.bias", "encoder.up_embed.out.1.weight",
            "encoder.up_embed.out.1.bias", "encoder.after_norm.weight", "encoder.after_norm.bias",
            "encoder_proj.weight", "encoder_proj.bias"]
E_LAYER = ["self_attn.linear_q.weight", "self_attn.linear_q.bias", "self_attn.linear_k.weight",
           "self_attn.linear_k.bias", "self_attn.linear_v.weight", "self_attn.linear_v.bias",
           "self_attn.linear_out.weight", "self_attn.linear_out.bias", "self_attn.linear_pos.weight",
           "self_attn.pos_bias_u", "self_attn.pos_bias_v", "feed_forward.w_1.weight", "feed_forward.w_1.bias",
           "feed_forward.w_2.weight", "feed_forward.w_2.bias", "norm_mha.weight", "norm_mha.bias", "norm_ff.weight",
           "norm_ff.bias"]


class HiftConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("mel", "channels", "f0_channels", "f0_layers", "harmonics", "sample_rate",
                                              "n_fft", "hop")] + \
               [(n, ctypes.c_int32 * 3) for n in ("up_rates", "up_kernels", "res_kernels", "source_kernels", "dilations")] + \
               [(n, ctypes.c_float) for n in ("nsf_alpha", "nsf_sigma", "voiced_threshold", "lrelu_slope", "audio_limit")] + \
               [("tf32", ctypes.c_int32), ("tf32_parts", ctypes.c_uint32)]


class VocodeBatch(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_int32), ("handle", ctypes.POINTER(ctypes.c_int32)),
                ("T", ctypes.POINTER(ctypes.c_int32)), ("last", ctypes.POINTER(ctypes.c_uint8))] + \
               [(n, ctypes.c_void_p) for n in ("mel", "rand_ini", "noise", "out", "source", "speech")] + \
               [("flags", ctypes.c_uint32), ("noise_ready", ctypes.c_void_p)]


class TConvArgs(ctypes.Structure):
    _fields_ = [("A", ctypes.c_void_p), ("lda", ctypes.c_int32), ("rows_a", ctypes.c_int32), ("W", ctypes.c_void_p),
                ("bias", ctypes.c_void_p)] + \
               [(n, ctypes.c_int32) for n in ("M", "N", "Cin", "taps", "tap_row0", "dil")] + \
               [("out", ctypes.c_void_p), ("ldo", ctypes.c_int64), ("row_mul", ctypes.c_int32),
                ("row_add", ctypes.c_int32), ("pad", ctypes.c_void_p), ("epi", ctypes.c_int32),
                ("alpha", ctypes.c_void_p), ("inv", ctypes.c_void_p), ("out2", ctypes.c_void_p),
                ("split_in", ctypes.c_int32), ("split_out", ctypes.c_int32), ("err", ctypes.c_void_p),
                ("resid_in", ctypes.c_void_p)]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_F = ctypes.c_float
_SIGS = {
    "t2w_version": ([], ctypes.c_int),
    "t2w_device_ok": ([ctypes.c_int], ctypes.c_int),
    "t2w_last_cuda_error": ([], ctypes.c_int),
    "t2w_create": ([ctypes.POINTER(Config), ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_P), _I, _I, _P,
                    ctypes.POINTER(_P)], ctypes.c_int),
    "t2w_destroy": ([_P], ctypes.c_int),
    "t2w_workspace_bytes": ([_P, _I, ctypes.POINTER(_I), ctypes.POINTER(_I)], ctypes.c_size_t),
    "t2w_solve_packed": ([_P, ctypes.POINTER(Batch), _P, ctypes.c_size_t, ctypes.c_uint32, _P], ctypes.c_int),
    "t2w_check": ([_P], ctypes.c_int),
    "t2w_test_wait_timeout": ([_P, ctypes.c_int64, _P], ctypes.c_int),
    "t2w_profile_solve": ([_P, ctypes.POINTER(Batch), _P, ctypes.c_size_t, _P, ctypes.POINTER(ctypes.c_float),
                           ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "t2w_mods": ([_P, _P, _P, _P, _P], ctypes.c_int),
    "t2w_counts": ([_P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)],
                   ctypes.c_int),
    "t2w_ln_mod": ([_P, _I, _P, _P, _F, _I, _I, _P, _I, _P, _P], ctypes.c_int),
    "t2w_add_ln_mod": ([_P, _P, _P, _P, _P, _F, _I, _I, _P, _P, _P], ctypes.c_int),
    "t2w_ln_mish": ([_P, _P, _P, _F, _I, _I, _P, _P, _P], ctypes.c_int),
    "t2w_gemm": ([_P, _I, _I, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I, ctypes.POINTER(_P), _F, _P], ctypes.c_int),
    "t2w_attn_varlen": ([_P, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I), _P, _P], ctypes.c_int),
    "t2w_attn_varlen_noalloc": ([_P, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I), _P, _P],
                                ctypes.c_int),
    "t2w_euler_cfg": ([_P, _P, _I, _P, _I, _I, _I, _F, _F, _P, _I, _P, _P], ctypes.c_int),
    "t2w_slots_create": ([_P, _I, _I, ctypes.POINTER(_P)], ctypes.c_int),
    "t2w_slots_destroy": ([_P], ctypes.c_int),
    "t2w_slots_copy": ([_P, ctypes.POINTER(_I), ctypes.POINTER(_I), _I, _P], ctypes.c_int),
    "t2w_slots_copy_row": ([_P, _I, _I, _P], ctypes.c_int),
    "t2w_slots_pools": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_I), ctypes.POINTER(_I),
                         ctypes.POINTER(_I), ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_slot_workspace_bytes": ([_P, _P, ctypes.POINTER(SlotBatch)], ctypes.c_size_t),
    "t2w_solve_slots": ([_P, _P, ctypes.POINTER(SlotBatch), _P, ctypes.c_size_t, ctypes.c_uint32, _P], ctypes.c_int),
    "t2w_cache_new": ([_P, _I, _P, ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_cache_release": ([_P, _I], ctypes.c_int),
    "t2w_cache_clone": ([_P, _I, _P, ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_cache_get": ([_P, _I, ctypes.POINTER(CacheInfo)], ctypes.c_int),
    "t2w_cache_set_keep": ([_P, _I, _I], ctypes.c_int),
    "t2w_cache_keys": ([_P, _I, _I, ctypes.POINTER(_I), _I], ctypes.c_int),
    "t2w_cache_reserve": ([_P, _I, _I, ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_slots_usage": ([_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_cached_workspace_bytes": ([_P, _P, ctypes.POINTER(CachedBatch)], ctypes.c_size_t),
    "t2w_solve_cached": ([_P, _P, ctypes.POINTER(CachedBatch), _P, ctypes.c_size_t, ctypes.c_uint32, _P], ctypes.c_int),
    "t2w_e4m3_sf_bytes": ([_I, _I], ctypes.c_size_t),
    "t2w_quant_e4m3": ([_P, _I, _I, _P, _P, _I, ctypes.c_int64, _P], ctypes.c_int),
    "t2w_quant_weight_e4m3": ([_P, _I, _I, _P, _P, _P], ctypes.c_int),
    "t2w_add_ln_mod_e4m3": ([_P, _P, _P, _P, _P, _F, _I, _I, _P, _P, _I, ctypes.c_int64, _P, _P], ctypes.c_int),
    "t2w_ln_mish_e4m3": ([_P, _P, _P, _F, _I, _I, _P, _P, _I, ctypes.c_int64, _P, _P], ctypes.c_int),
    "t2w_attn_varlen_e4m3": ([_P, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I), _P, _P, _P],
                             ctypes.c_int),
    "t2w_encoder_create": ([ctypes.POINTER(EncConfig), ctypes.POINTER(_P), _I, _I, _I, _I, _I, _P, ctypes.POINTER(_P)],
                           ctypes.c_int),
    "t2w_encoder_destroy": ([_P], ctypes.c_int),
    "t2w_enc_stream_new": ([_P, _I, _P, ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_enc_stream_release": ([_P, _I], ctypes.c_int),
    "t2w_enc_stream_clone": ([_P, _I, _P, ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_enc_stream_get": ([_P, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_enc_usage": ([_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_enc_workspace_bytes": ([_P, ctypes.POINTER(EncBatch)], ctypes.c_size_t),
    "t2w_encode": ([_P, ctypes.POINTER(EncBatch), _P, ctypes.c_size_t, ctypes.c_uint32, _P], ctypes.c_int),
    "t2w_enc_counts": ([_P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                        ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "t2w_enc_check": ([_P], ctypes.c_int),
    "t2w_enc_relattn": ([_P, _I, _I, _P, _I, _P, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                         ctypes.POINTER(_I), ctypes.POINTER(_I), _I, _P, _P], ctypes.c_int),
    "t2w_enc_pos_table": ([_P, _I, _I, _F, _P, _P], ctypes.c_int),
    "t2w_enc_ln": ([_P, _P, _P, _F, _I, _I, _P, _P, _P, _P], ctypes.c_int),
    "t2w_hift_create": ([ctypes.POINTER(HiftConfig), ctypes.POINTER(_P), _I, _I, _I, ctypes.POINTER(_P)], ctypes.c_int),
    "t2w_hift_destroy": ([_P], ctypes.c_int),
    "t2w_hift_check": ([_P], ctypes.c_int),
    "t2w_hift_stream_new": ([_P, ctypes.POINTER(_I)], ctypes.c_int),
    "t2w_hift_stream_release": ([_P, _I], ctypes.c_int),
    "t2w_vocode_samples": ([_P, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_uint8),
                            ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(_I)], ctypes.c_int64),
    "t2w_vocode": ([_P, ctypes.POINTER(VocodeBatch), _P], ctypes.c_int),
    "t2w_test_tconv": ([ctypes.POINTER(TConvArgs), _P], ctypes.c_int),
    "t2w_test_attn_gathered": ([_P, _I, _I, _I, ctypes.POINTER(_I), _P, _I, _I, ctypes.POINTER(_I), _I, _I, _P, _P, _P],
                               ctypes.c_int),
    "t2w_hift_counts": ([_P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                         ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "t2w_gemm_e4m3": ([_P, _I, _I, _P, _I, ctypes.c_int64, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _P,
                       ctypes.POINTER(_P), _F, _P], ctypes.c_int),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function the public headers declare."""
    out = []
    for f in sorted(os.listdir(INCLUDE)):
        if f.endswith(".h"):
            src = open(os.path.join(INCLUDE, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            out += re.findall(r"^\s*(?:T2W_API\s+)?(?:size_t|int64_t|int|void)\s+(t2w_\w+)\s*\(", src, flags=re.M)
    return out


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and type the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        path = path or LIB_PATH
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with b200t2w.build.build()")
        lib = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = args, res
        _lib = lib
    return _lib


def check(fn: str, status: int) -> None:
    if status != T2W_OK:
        raise T2WError(fn, status, load().t2w_last_cuda_error() if status == -2 else 0)


def call(fn: str, *args) -> int:
    rc = getattr(load(), fn)(*args)
    check(fn, rc)
    return rc


def i32_array(xs) -> ctypes.Array:
    return (ctypes.c_int32 * len(xs))(*[int(x) for x in xs])
