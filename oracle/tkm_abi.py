"""ctypes mirror of the public structs of include/tkm.h (TkmGraph and its
members), used by the tests to compare node tables field by field."""
import ctypes as C

MAX_NODES, MAX_GROUPS, MAX_CHAIN, MAX_KARGS = 1024, 256, 8, 28


class KernelArg(C.Structure):
    _fields_ = [("kind", C.c_int), ("node_id", C.c_int), ("c_type", C.c_char * 32), ("c_name", C.c_char * 32)]


class KernelSig(C.Structure):
    _fields_ = [("func_name", C.c_char * 64), ("args", KernelArg * MAX_KARGS), ("num_args", C.c_int),
                ("grid_x", C.c_int), ("block_x", C.c_int)]


class Node(C.Structure):
    _fields_ = [
        ("id", C.c_int), ("spec_id", C.c_int), ("tag", C.c_char * 32), ("op", C.c_int), ("cat", C.c_int),
        ("dead", C.c_int), ("in0", C.c_int), ("in1", C.c_int), ("in2", C.c_int), ("users", C.c_int),
        ("plasma_grp", C.c_int), ("c_out", C.c_int), ("k", C.c_int), ("s", C.c_int), ("p", C.c_int),
        ("q_c", C.c_int), ("k_c", C.c_int), ("v_c", C.c_int), ("q_heads", C.c_int), ("kv_heads", C.c_int),
        ("head_dim", C.c_int), ("has_qknorm", C.c_int), ("has_rope", C.c_int), ("causal", C.c_int),
        ("qkv_prep_nid", C.c_int), ("fval", C.c_float), ("fval2", C.c_float), ("rope_theta", C.c_float),
        ("rope_scale", C.c_float), ("rope_low_freq_factor", C.c_float), ("rope_high_freq_factor", C.c_float),
        ("rope_original_context_length", C.c_float), ("rng_type", C.c_int),
        ("left_nodes", C.c_int * MAX_CHAIN), ("left_len", C.c_int), ("right_nodes", C.c_int * MAX_CHAIN),
        ("right_len", C.c_int), ("H", C.c_int), ("W", C.c_int), ("C", C.c_int), ("out_buf_id", C.c_int),
        ("out_offset", C.c_size_t), ("out_bytes", C.c_size_t),
    ]


class Group(C.Structure):
    _fields_ = [
        ("id", C.c_int), ("anchor_id", C.c_int), ("node_ids", C.c_int * 16), ("count", C.c_int),
        ("has_norm", C.c_int), ("is_twin_epilogue", C.c_int), ("is_coord_group", C.c_int),
        ("is_qkv_prep", C.c_int), ("use_reflect_border", C.c_int), ("out_node_id", C.c_int),
        ("H", C.c_int), ("W", C.c_int), ("C", C.c_int), ("fwd_sig", KernelSig), ("bwd_sig", KernelSig),
    ]


class Graph(C.Structure):
    _fields_ = [("nodes", Node * MAX_NODES), ("num_nodes", C.c_int), ("groups", Group * MAX_GROUPS),
                ("num_groups", C.c_int), ("batch_size", C.c_int), ("default_rng", C.c_int),
                ("total_arena_bytes", C.c_size_t), ("naive_arena_bytes", C.c_size_t)]


class OpSpec(C.Structure):
    _fields_ = [("op", C.c_int), ("dsl_name", C.c_char_p), ("cat", C.c_int), ("res_flags", C.c_uint32),
                ("default_fval", C.c_float), ("fwd_cuda", C.c_char_p), ("bwd_cuda", C.c_char_p),
                ("fwd_expr", C.c_char_p), ("bwd_expr", C.c_char_p)]


def bind(lib):
    """Declare the compiler-API signatures on a loaded libtkm (ours or the reference's)."""
    G = C.POINTER(Graph)
    lib.tkm_parse_dsl.argtypes = [G, C.c_char_p, C.c_int]
    lib.tkm_parse_dsl.restype = None
    lib.tkm_optimize_and_bind.argtypes = [G]
    lib.tkm_optimize_and_bind.restype = None
    lib.tkm_infer_shapes.argtypes = [G]
    lib.tkm_infer_shapes.restype = None
    lib.tkm_plan_memory.argtypes = [G]
    lib.tkm_plan_memory.restype = None
    lib.tkm_codegen_cuda_string.argtypes = [G]
    lib.tkm_codegen_cuda_string.restype = C.c_void_p
    lib.tkm_verify_registry.argtypes = []
    lib.tkm_verify_registry.restype = C.c_int
    lib.tkm_get_spec_count.argtypes = []
    lib.tkm_get_spec_count.restype = C.c_int
    lib.tkm_find_spec_by_index.argtypes = [C.c_int]
    lib.tkm_find_spec_by_index.restype = C.POINTER(OpSpec)
    lib.tkm_eval_math_expr.argtypes = [C.c_char_p, C.c_float, C.c_float, C.POINTER(C.c_float)]
    lib.tkm_eval_math_expr.restype = C.c_int
    lib.tkm_get_fusion_rules.argtypes = [C.POINTER(C.c_int)]
    lib.tkm_get_fusion_rules.restype = C.c_void_p
    lib.tkm_rng_name.argtypes = [C.c_int]
    lib.tkm_rng_name.restype = C.c_char_p
    lib.tkm_parse_rng_name.argtypes = [C.c_char_p]
    lib.tkm_parse_rng_name.restype = C.c_int
    return lib


def compile_graph(lib, dsl, batch):
    g = Graph()
    lib.tkm_parse_dsl(C.byref(g), dsl.encode(), batch)
    lib.tkm_optimize_and_bind(C.byref(g))
    lib.tkm_plan_memory(C.byref(g))
    return g
