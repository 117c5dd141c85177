"""ctypes bindings of the C ABI in include/d1kernels.h and include/d1h.h.

The struct layouts mirror the reference's repr(C) types (src/cuda.rs:59-100) and the runner's weight structs;
`bind(lib)` attaches argument/return types to every exported function of a loaded library so a wrong argument
count or type fails in Python instead of on the GPU.
"""
import ctypes as C

p = C.c_void_p
i32 = C.c_int
f32 = C.c_float


class SeqInfo(C.Structure):
    """cuda/kernels.cu:15-24, src/cuda.rs:59-70 (48 bytes)."""
    _fields_ = [("start", i32), ("len", i32), ("pos_off", i32), ("qtype", i32),
                ("ext_bx", p), ("save_bx", p), ("save_k", p), ("save_v", p)]


class AttnSeq(C.Structure):
    """cuda/kernels.cu:26-32, src/cuda.rs:88-99 (40 bytes)."""
    _fields_ = [("q_start", i32), ("q_len", i32), ("kv_start", i32), ("kv_len", i32),
                ("ext_len", i32), ("_pad", i32), ("ext_k", p), ("ext_v", p)]


assert C.sizeof(SeqInfo) == 48 and C.sizeof(AttnSeq) == 40


class TrunkLayer(C.Structure):
    _fields_ = [("is_attn", i32), ("in_proj", p), ("out_proj", p), ("convw", p), ("qkv", p), ("out", p),
                ("qn", p), ("kn", p), ("op_norm", p), ("ffn_norm", p), ("gate_up", p), ("down", p), ("ffn", i32)]


class HeadLayer(C.Structure):
    _fields_ = [("n1_w", p), ("n1_b", p), ("qkv", p), ("qkv_b", p), ("out", p), ("out_b", p), ("n2_w", p),
                ("n2_b", p), ("up", p), ("up_b", p), ("down", p), ("down_b", p), ("ffn", i32)]


class TextWeights(C.Structure):
    _fields_ = [("n_layers", i32), ("layers", C.POINTER(TrunkLayer)), ("n_head", i32),
                ("head", C.POINTER(HeadLayer)), ("vocab", i32), ("embed", p), ("final_norm", p),
                ("type_emb", p), ("cls_norm_w", p), ("cls_norm_b", p), ("cls_w", p), ("cls_b", p), ("out_w", p),
                ("out_b", f32), ("eps", f32), ("rope_theta", f32)]


class VisionLayer(C.Structure):
    _fields_ = [("ln1_w", p), ("ln1_b", p), ("qkv", p), ("qkv_b", p), ("out", p), ("out_b", p), ("ln2_w", p),
                ("ln2_b", p), ("fc1", p), ("fc1_b", p), ("fc2", p), ("fc2_b", p)]


class VisionWeights(C.Structure):
    _fields_ = [("n_layers", i32), ("layers", C.POINTER(VisionLayer)), ("patch_w", p), ("patch_b", p), ("pos", p),
                ("post_w", p), ("post_b", p), ("proj1", p), ("proj1_b", p), ("proj2", p), ("proj2_b", p),
                ("eps", f32)]


class PrefixCache(C.Structure):
    _fields_ = [("len", i32), ("k", p), ("v", p), ("bx", p)]


class TextSeq(C.Structure):
    _fields_ = [("ids", C.POINTER(i32)), ("n_ids", i32), ("markers", C.POINTER(i32)), ("n_markers", i32),
                ("qtype", i32), ("prefix", C.POINTER(PrefixCache))]


class PrefixSeq(C.Structure):
    _fields_ = [("emb", p), ("cache", C.POINTER(PrefixCache))]


class AudioLayer(C.Structure):
    _fields_ = [("ff1_n_w", p), ("ff1_n_b", p), ("ff1_up", p), ("ff1_up_b", p), ("ff1_down", p), ("ff1_down_b", p),
                ("att_n_w", p), ("att_n_b", p), ("qkv", p), ("bq", p), ("bk", p), ("bv", p), ("pu", p), ("pv", p),
                ("pos", p), ("out", p), ("out_b", p), ("conv_n_w", p), ("conv_n_b", p), ("pw1", p), ("pw1_b", p),
                ("dw", p), ("dw_b", p), ("bn_s", p), ("bn_b", p), ("pw2", p), ("pw2_b", p), ("ff2_n_w", p),
                ("ff2_n_b", p), ("ff2_up", p), ("ff2_up_b", p), ("ff2_down", p), ("ff2_down_b", p), ("out_n_w", p),
                ("out_n_b", p)]


class AudioWeights(C.Structure):
    _fields_ = [("n_layers", i32), ("layers", C.POINTER(AudioLayer)), ("c0_w", p), ("c0_b", p), ("c2_w", p),
                ("c2_b", p), ("c3_w", p), ("c3_b", p), ("c5_w", p), ("c5_b", p), ("c6_w", p), ("c6_b", p),
                ("pre_out", p), ("pre_out_b", p), ("ad_n_w", p), ("ad_n_b", p), ("ad1", p), ("ad1_b", p), ("ad2", p),
                ("ad2_b", p), ("res_n_w", p), ("res_n_b", p), ("res_down", p), ("res_down_b", p), ("res_up", p),
                ("res_up_b", p), ("eps", f32)]



class EngineConfig(C.Structure):
    _fields_ = [("max_batch_tokens", i32), ("cap_tokens", i32), ("media_cache_bytes", C.c_longlong)]


class Row(C.Structure):
    _fields_ = [("ids", C.POINTER(i32)), ("n_ids", i32), ("markers", C.POINTER(i32)), ("n_markers", i32),
                ("qtype", i32)]


class Media(C.Structure):
    _fields_ = [("kind", i32), ("n_crops", i32), ("ph", C.POINTER(i32)), ("pw", C.POINTER(i32)), ("patches", p),
                ("mel", C.POINTER(f32)), ("valid", i32), ("pcm", C.POINTER(f32)), ("n_samples", i32),
                ("sample_rate", i32)]


class Job(C.Structure):
    _fields_ = [("rows", C.POINTER(Row)), ("n_rows", i32), ("media", Media)]


class EngineStats(C.Structure):
    _fields_ = [("tokens", C.c_longlong), ("media_tokens", C.c_longlong), ("batches", C.c_longlong),
                ("media_jobs", C.c_longlong), ("rows", C.c_longlong)]


# name -> (restype, argtypes). The kernel ABI (d1kernels.h) first, then the runner (d1h.h).
KERNELS = {
    "d1_rmsnorm": (i32, [p, p, p, i32, i32, f32, p]),
    "d1_layernorm": (i32, [p, p, f32, p, p, p, p, i32, i32, f32, p]),
    "d1_head_init": (i32, [p, p, p, p, p, p, i32, f32, p]),
    "d1_embed": (i32, [p, p, p, i32, i32, p]),
    "d1_swiglu": (i32, [p, p, i32, i32, p]),
    "d1_bias_act_h": (i32, [p, p, i32, i32, i32, p]),
    "d1_bias_act_f": (i32, [p, p, i32, i32, i32, p]),
    "d1_fill_rows": (i32, [p, p, p, i32, i32, p]),
    "d1_f32_to_f16": (i32, [p, p, C.c_size_t, p]),
    "d1_gather_rows": (i32, [p, p, p, i32, i32, p]),
    "d1_shortconv": (i32, [p, p, p, p, p, i32, i32, i32, p]),
    "d1_qk_norm_rope": (i32, [p, i32, i32, i32, p, p, p, p, p, i32, i32, f32, p]),
    "d1_flash_attn": (i32, [p, i32, p, p, i32, i32, p, p, p, p, i32, p, p, i32, i32, i32, f32, p]),
    "d1_scorer_out": (i32, [p, p, p, f32, p, i32, i32, p]),
    "d1_unshuffle": (i32, [p, p, i32, i32, i32, p]),
    "d1_sub_conv0": (i32, [p, i32, i32, p, p, p, i32, i32, p]),
    "d1_sub_dwconv": (i32, [p, i32, i32, p, p, p, i32, i32, p]),
    "d1_relpos_prep": (i32, [p, p, p, p, p, p, p, p, p, p, i32, i32, p]),
    "d1_relpos_softmax": (i32, [p, p, p, i32, i32, f32, p]),
    "d1_conformer_dw": (i32, [p, p, p, p, p, p, p, i32, i32, i32, p]),
    "d1_lt_init": (p, [C.c_size_t]),
    "d1_lt_gemm": (i32, [p, i32, i32, i32, p, i32, p, i32, i32, p, i32, i32, i32, f32, f32, p]),
    "d1_lt_tune": (f32, [p, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, p]),
    "d1_lt_save": (i32, [p, C.c_char_p]),
    "d1_lt_load": (i32, [p, C.c_char_p]),
    "d1_lt_bucket": (i32, [i32]),
    "d1_lt_free_scratch": (None, [p]),
}

EXTENSIONS = {
    "d1_gemm_swiglu": (i32, [p, i32, i32, i32, p, i32, p, i32, p, i32, p]),
    "d1_gemm_bias_act": (i32, [p, i32, i32, i32, p, i32, p, i32, p, i32, p, i32, p]),
    "d1_gemm_qk_norm_rope": (i32, [p, i32, i32, p, i32, p, i32, p, i32, i32, i32, p, p, p, p, p, f32, p]),
    "d1_lt_error": (i32, [p]),
    "d1_flash_attn_error": (i32, []),
    "d1_flash_attn_tc": (i32, [p, i32, p, p, i32, i32, p, i32, p, p, i32, i32, i32, f32, i32, i32, p]),
    "d1_sgemm": (i32, [i32, i32, i32, p, i32, p, i32, p, i32, f32, p, i32, p]),
    "d1_relpos_attn": (i32, [p, p, p, p, i32, p, i32, i32, i32, p, i32, p, i32, i32, i32, f32, p]),
    "d1_relpos_attn_error": (i32, []),
    "d1_log_mel": (i32, [p, i32, p, p]),
    "d1_resample_len": (i32, [i32, i32, i32]),
    "d1_resample": (i32, [p, i32, i32, i32, p, p]),
    "d1_vision_pos": (i32, [p, p, p, p, i32, i32, i32, i32, p, p]),
    "d1_layernorm_rows": (i32, [p, p, f32, p, p, p, p, i32, i32, f32, p]),
    "d1_sub_conv01": (i32, [p, i32, i32, p, p, p, p, p, i32, i32, p]),
    "d1_conformer_dw_clips": (i32, [p, p, p, p, p, p, p, p, i32, i32, i32, i32, p]),
    "d1_gemm_noalloc": (i32, [i32, i32, i32, p, i32, p, i32, p, i32, i32, p]),
    "d1_gemm_noalloc_error": (i32, []),
    "d1_lt_destroy": (None, [p]),
    "d1_build_id": (C.c_char_p, []),
}

RUNNER = {
    "d1h_model_create": (p, [C.POINTER(TextWeights), C.c_char_p, i32]),
    "d1h_model_destroy": (None, [p]),
    "d1h_last_error": (C.c_char_p, []),
    "d1h_workspace_create": (p, [p, i32]),
    "d1h_workspace_destroy": (None, [p]),
    "d1h_launch_text": (i32, [p, p, i32, C.POINTER(TextSeq), i32, p]),
    "d1h_finish": (i32, [p, p, i32, C.POINTER(f32), i32]),
    "d1h_prefix_alloc": (i32, [p, i32, C.POINTER(PrefixCache), p]),
    "d1h_prefix_free": (None, [C.POINTER(PrefixCache), p]),
    "d1h_launch_prefix": (i32, [p, p, i32, C.POINTER(PrefixSeq), i32, p]),
    "d1h_tune": (i32, [p, p, i32, p]),
    "d1h_launch_count": (C.c_longlong, [p]),
    "d1h_h2d_bytes": (C.c_longlong, [p, i32]),
    "d1h_vision_create": (p, [C.POINTER(VisionWeights), C.c_char_p, i32, i32]),
    "d1h_vision_destroy": (None, [p]),
    "d1h_vision_encode": (i32, [p, i32, C.POINTER(i32), C.POINTER(i32), p, p, p]),
    "d1h_d2h_bytes": (C.c_longlong, [p, i32]),
    "d1h_audio_create": (p, [C.POINTER(AudioWeights), i32, i32]),
    "d1h_audio_destroy": (None, [p]),
    "d1h_audio_encode": (i32, [p, i32, C.POINTER(i32), p, p, p]),
    "d1h_audio_encode_pcm": (i32, [p, i32, C.POINTER(i32), p, p, C.POINTER(i32), p]),
    "d1h_audio_encode_pcm_rates": (i32, [p, i32, C.POINTER(i32), C.POINTER(i32), p, p, C.POINTER(i32), p]),
    "d1h_vision_capacity": (i32, [p]),
    "d1h_model_layers": (i32, [p, i32]),
    "d1h_gemm_ctx": (p, [p]),
    "d1h_set_tune_effort": (i32, [p, i32]),
    "d1e_create": (p, [p, p, p, C.POINTER(EngineConfig), p]),
    "d1e_destroy": (None, [p]),
    "d1e_submit": (C.c_longlong, [p, C.POINTER(Job)]),
    "d1e_step": (i32, [p]),
    "d1e_pending": (i32, [p]),
    "d1e_queued_tokens": (C.c_longlong, [p]),
    "d1e_next_logits": (i32, [p]),
    "d1e_take": (i32, [p, C.POINTER(C.c_longlong), C.POINTER(f32), i32, C.c_char_p, i32]),
    "d1e_stats": (None, [p, C.POINTER(EngineStats)]),
    "d1e_last_error": (C.c_char_p, []),
}


def bind(lib, tables=(KERNELS, EXTENSIONS, RUNNER), required=True):
    """Attach prototypes; returns the names that are missing from the library."""
    missing = []
    for table in tables:
        for name, (res, args) in table.items():
            fn = getattr(lib, name, None)
            if fn is None:
                missing.append(name)
                continue
            fn.restype = res
            fn.argtypes = args
    if required and missing:
        raise RuntimeError(f"library {lib._name} lacks {missing}")
    return missing
