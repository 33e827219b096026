"""ctypes declarations of the training-step C ABI (include/llmgpu.h)."""
import ctypes

c_int, c_ll, c_vp, c_float, c_size_t, c_char_p = (ctypes.c_int, ctypes.c_longlong,
                                                  ctypes.c_void_p, ctypes.c_float,
                                                  ctypes.c_size_t, ctypes.c_char_p)
P_i32 = ctypes.POINTER(ctypes.c_int32)
P_f32 = ctypes.POINTER(ctypes.c_float)
P_i64 = ctypes.POINTER(ctypes.c_int64)
P_int = ctypes.POINTER(ctypes.c_int)


class LlmgpuConfig(ctypes.Structure):
    _fields_ = [("vocab_size", c_int), ("n_layers", c_int), ("n_heads", c_int),
                ("n_embd", c_int), ("block_size", c_int), ("weight_tying", c_int),
                ("use_rmsnorm", c_int), ("use_mamba", c_int), ("d_inner", c_int),
                ("d_state", c_int), ("dt_rank", c_int), ("conv_kernel", c_int),
                ("ffn_swiglu", c_int), ("ffn_hidden", c_int), ("rope_qk", c_int),
                ("rope_theta", c_float), ("moe_experts", c_int), ("moe_top_k", c_int),
                ("moe_aux_coef", c_float), ("pos_encoding", c_int), ("rope_scaling", c_float),
                ("rope_mode", c_int), ("yarn_alpha", c_float), ("yarn_beta", c_float)]


SIGS = {
    "llmgpu_config_default": ([ctypes.POINTER(LlmgpuConfig)], None),
    "llmgpu_get_unique_id": ([c_vp], c_int),
    "llmgpu_create": ([ctypes.POINTER(LlmgpuConfig), c_int, c_int, c_int, c_int, c_vp], c_vp),
    "llmgpu_destroy": ([c_vp], c_int),
    "llmgpu_last_error": ([c_vp], c_char_p),
    "llmgpu_set_adamw": ([c_vp, c_float, c_float, c_float, c_float, c_float], c_int),
    "llmgpu_set_lr": ([c_vp, c_float], c_int),
    "llmgpu_set_train": ([c_vp, c_float, c_int, c_float], c_int),
    "llmgpu_set_loss_scale": ([c_vp, c_float], c_int),
    "llmgpu_set_comm_timeout": ([c_vp, ctypes.c_double], c_int),
    "llmgpu_abort_comm": ([c_vp], c_int),
    "llmgpu_train_step": ([c_vp, P_i32, c_int, c_int, P_f32, P_f32], c_int),
    "llmgpu_train_step_accum": ([c_vp, P_i32, c_int, c_int, P_f32, P_int], c_int),
    "llmgpu_train_step_device": ([c_vp, c_vp, c_int, c_int, P_f32, P_f32], c_int),
    "llmgpu_eval_loss": ([c_vp, P_i32, c_int, c_int, P_f32], c_int),
    "llmgpu_forward_logits": ([c_vp, P_i32, c_int, c_int, P_f32, ctypes.c_int64], ctypes.c_int64),
    "llmgpu_forward_logits_all": ([c_vp, P_i32, c_int, c_int, P_f32, ctypes.c_int64],
                                  ctypes.c_int64),
    "llmgpu_decode_reset": ([c_vp, c_int], c_int),
    "llmgpu_decode_prefill": ([c_vp, P_i32, c_int, c_int, P_f32, ctypes.c_int64], ctypes.c_int64),
    "llmgpu_decode_step": ([c_vp, P_i32, c_int, P_f32, ctypes.c_int64], ctypes.c_int64),
    "llmgpu_decode_position": ([c_vp], c_int),
    "llmgpu_num_params": ([c_vp], c_int),
    "llmgpu_num_parameters": ([c_vp], c_size_t),
    "llmgpu_param_info": ([c_vp, c_int, c_char_p, c_int, P_i64], c_int),
    "llmgpu_get_param": ([c_vp, c_int, P_f32, ctypes.c_int64], ctypes.c_int64),
    "llmgpu_get_grad": ([c_vp, c_int, P_f32, ctypes.c_int64], ctypes.c_int64),
    "llmgpu_get_adam_state": ([c_vp, c_int, P_f32, P_f32, ctypes.c_int64], ctypes.c_int64),
    "llmgpu_set_param": ([c_vp, c_int, P_f32, ctypes.c_int64], c_int),
    "llmgpu_save_binary": ([c_vp, c_char_p], c_int),
    "llmgpu_load_binary": ([c_vp, c_char_p], c_int),
    "llmgpu_save_train_state": ([c_vp, c_char_p], c_int),
    "llmgpu_load_train_state": ([c_vp, c_char_p], c_int),
    "llmgpu_step": ([c_vp], c_int),
    "llmgpu_set_step": ([c_vp, c_int], c_int),
    "llmgpu_skipped_steps": ([c_vp], c_int),
    "llmgpu_last_loss": ([c_vp], c_float),
    "llmgpu_last_grad_norm": ([c_vp], c_float),
    "llmgpu_last_timings": ([c_vp, P_f32], c_int),
    "llmgpu_last_launches": ([c_vp], c_int),
    "llmgpu_set_graph": ([c_vp, c_int], c_int),
    "llmgpu_stream": ([c_vp], c_vp),
    "llmgpu_set_profile": ([c_vp, c_int], c_int),
    "llmgpu_gemm_stats": ([c_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                           P_int, c_int], c_int),
    "llmgpu_gemm_last_step": ([c_vp, P_i32, P_f32, c_int], c_int),
    "llmgpu_moe_routing": ([c_vp, c_int, P_i32, ctypes.c_int64], ctypes.c_int64),
}


def declare(lib):
    for name, (args, res) in SIGS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
