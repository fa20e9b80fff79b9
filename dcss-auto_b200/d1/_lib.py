"""ctypes loader for libd1.so with argument types for every exported entry point."""
import ctypes as C
import pathlib

LIB_PATH = pathlib.Path(__file__).resolve().parent / 'libd1.so'
ERR_NO_HOST_PATH = 9001
ERR_BAD_ARGUMENT = 9002
ERR_TOO_LARGE = 9003

_P, _I, _U64, _F = C.c_void_p, C.c_int, C.c_uint64, C.c_float
# name -> argtypes; every export returns int.
SIGNATURES = {
    'learn_state_bytes': [], 'learn_obs_size': [], 'learn_action_size': [], 'learn_out_size': [],
    'learn_config_bytes': [],
    'learn_init': [_P, _I, _P, _P, _U64, _P, _P, _P, _I],
    'learn_step': [_P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _I],
    'learn_step_active': [_P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I],
    'learn_heuristic': [_P, _I, _P, _P, _P, _P, _I],
    'learn_semantic_test': [_P, _P],
    'learn_compact_state': [_P, _I, _P, _P],
    'learn_distance_table': [_P, _P, _I, _P, _P],
    'd1_spec_state_bytes': [], 'd1_spec_obs_size': [], 'd1_spec_action_size': [], 'd1_spec_out_size': [],
    'd1_spec_config_bytes': [],
    'd1_spec_set_rays': [_P, _I],
    'd1_spec_init': [_P, _I, _P, _U64, _I, _P, _P, _P],
    'd1_spec_step': [_P, _I, _P, _P, _P, _P, _P, _P, _P],
    'd1_spec_init_ex': [_P, _I, _P, _U64, _I, _P, _P, _P, _P],
    'd1_spec_step_ex': [_P, _I, _P, _P, _P, _P, _P, _P, _P, _P],
    'd1_spec_step_strided': [_P, _I, _P, _P, _P, _P, _P, _P, C.c_int64, C.c_int64, _P, _P],
    'd1_ppo_gather_cobs': [_P, _P, _I, _P, _I, _I, _P],
    'd1_spec_compact': [_P, _I, _P, _P],
    'd1_spec_observe': [_P, _I, _P, _P, _P, _P, _P],
    'd1_spec_planes': [_P, _I, _P, _P, _P],
    'd1_policy_head_sample': [_P, _I, _I, _P, _P, _P, _U64, _U64, _I, _P, _P, _P, _P, _P],
    'd1_gemm': [_P, _I, _P, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _P],
    'd1_gae': [_P, _P, C.c_int64, C.c_int64, _P, _I, _I, _F, _F, _P, _P, _P, _I, _P],
    'd1_ppo_loss_part_len': [],
    'd1_ppo_loss': [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_double, _I, _F, _F, _F, _F, _P, _P, _I, _P, _I, _P],
    'd1_reduce_slabs': [_P, _I, C.c_int64, _P, _P],
    'd1_counter_add': [_P, C.c_int64, _P],
    'd1_ppo_permute': [_P, C.c_int64, C.c_uint64, _P, _P],
    'd1_ppo_tail': [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_double, _I, _F, _F, _F, _F, _P, _P, _P, _P],
    'd1_ppo_tail_blocks': [_I],
    'd1_ppo_tail_error': [],
    'd1_policy_tail_sample': [_P, _I, _I, _P, _P, _P, _P, _P, C.c_uint64, C.c_uint64, _P, _I, _P, _P, _P, _P, _P],
    'd1_policy_tail_error': [],
    'd1_gemm_splits': [_I, _I],
    'd1_gemm_bkn': [_P, _I, _P, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I, _I, _P],
    'd1_gemm_rows': [_P, _I, _I, _P, _I, _P, _I, _I, _P, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _P],
    'd1_gemm_ex': [_P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _P],
    'd1_gemm_single': [_P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _P],
    'd1_spec_d4_observe': [_P, _P, _P, _I, _P, _P, _P],
    'd1_spec_d4_actions': [_P, _P, _I, _P, _P],
    'd1_spec_d4_draw': [_P, _I, _P, _I, _P, _U64, _U64, _I, _P],
    'd1_ppo_step': [_P, _I, _P, _P, _P, _P, C.c_int64, _F, _F, _F, _F, _F, _P, _P, _I, _P],
    'd1_grad_reduce': [_P, _I, _P],
    'd1_ppo_step_peer': [_P, _I, _P, _P, _P, _P, C.c_int64, _F, _F, _F, _F, _F, _P, _P, _I, _P, _P, C.c_int64, _I,
                         _I, C.c_uint, _P],
    'd1_ppo_step_peer2': [_P, _I, _P, _P, _P, _P, C.c_int64, _F, _F, _F, _F, _F, _P, _P, _I, _P, _P, C.c_int64, _I,
                          _I, C.c_uint, _P],
    'd1_ppo_step_nvls': [_P, _I, _P, _P, _P, _P, C.c_int64, _F, _F, _F, _F, _F, _P, _P, _I, _P, _P, C.c_int64, _P,
                         _I, _I, C.c_uint, _P],
    'd1_peer_handle_bytes': [],
    'd1_peer_alloc': [C.c_int64, _P, _P],
    'd1_peer_open': [_P, _P],
    'd1_peer_close': [_P],
    'd1_peer_free': [_P],
    'd1_peer_error': [],
    'd1_ppo_gather_x': [_P, _I, _P, _I, _P, _I, _I, _P],
    'd1_gemm_cobs_a': [_P, _P, _I, _P, _I, _I, _P, _I, _P, _I, _P],
    'd1_gemm_cobs_b': [_P, _I, _P, _P, _I, _I, _I, _P, _I, _I, _P],
    'd1_gemm_pair': [_P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _P],
    'd1_gemm_head_sample': [_P, _I, _P, _I, _I, _I, _P, _P, _P, _P, _U64, _U64, _I, _P, _P, _P, _P, _P],
    'd1_gemm_error': [],
    'd1_gemm_wgrad_noalloc': [_P, _I, _P, _I, _I, _I, _I, _P, _I, _I, _P],
    'd1_spec_crop': [_P, _I, _I, _P, _P],
    'd1_los_table': [_P, _P, _P],
    'd1_conv_in_bytes': [_I],
    'd1_conv_weight_bytes': [_I],
    'd1_conv_pack_weights': [_I, _P, _P, _P],
    'd1_conv_layer': [_I, _P, _I, _P, _P, _P, _P],
    'd1_conv_error': [],
    'd1_ar_head_sample': [_P, _I, _P, _P, _P, _P, _U64, _U64, _I, _P, _P, _P, _P, _P, _P, _P, _P],
    'd1_ar_head_greedy': [_P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    'd1_policy_head_greedy': [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    'd1_policy_head_sample_dev': [_P, _I, _I, _P, _P, _P, _U64, _P, _I, _P, _P, _P, _P, _P],
    'd1_eval_accumulate': [_P, _I, _I, _P, _P, _P, _I, _P],
    'd1_sample_uniform_legal': [_P, _I, _I, _U64, _U64, _I, _P, _P],
    'd1_frame_stack': [_P, _P, _I, _I, _I, _P, _I, _P, _P],
    'd1_route_state_bytes': [], 'd1_route_obs_size': [], 'd1_route_action_size': [], 'd1_route_out_size': [],
    'd1_route_config_bytes': [], 'd1_route_compact_size': [],
    'd1_route_init': [_P, _I, _P, _P, _U64, _P, _P, _P, _P],
    'd1_route_step': [_P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P],
    'd1_route_heuristic': [_P, _I, _P, _P, _P, _P],
    'd1_route_observe': [_P, _I, _P, _P, _P, _P, _P, _P],
    'd1_route_compact': [_P, _I, _P, _P],
    'd1_route_memory': [_P, _I, _P, _P, _P],
}

_LIB = None


class D1Error(RuntimeError):
    pass


def library():
    """Load libd1.so once; raise (never fall back) when it is missing."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise D1Error(f'{LIB_PATH} is missing: build it with `make -C dcss-auto_b200/csrc` '
                          '(or __graft_entry__.build()); there is no CPU fallback')
        lib = C.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = C.c_int
        _LIB = lib
    return _LIB


def resolve_device(device):
    """A CUDA device with its index: 'cuda' (no index) is the current device,
    as in torch, so an object built after torch.cuda.set_device(r) lives on
    GPU r. libd1 launches on the current device with the pointers it is given,
    so an object's tensors and its launches must agree on the device."""
    import torch
    dev = torch.device(device)
    if dev.type != 'cuda':
        return dev
    return dev if dev.index is not None else torch.device('cuda', torch.cuda.current_device())


def launch_stream(device):
    """The current stream of `device` for a libd1 launch, after checking that
    `device` is the current CUDA device: libd1 launches on the current device,
    so pointers of another GPU would be read by the wrong one."""
    import torch
    dev = torch.device(device)
    cur = torch.cuda.current_device()
    if dev.index is not None and dev.index != cur:
        raise D1Error(f'tensors on {dev} but the current CUDA device is cuda:{cur}: '
                      f'call torch.cuda.set_device({dev.index}) (or use torch.cuda.device) first')
    return torch.cuda.current_stream(dev).cuda_stream


def check(code, what='libd1 call'):
    if code:
        raise D1Error(f'{what} failed with error {code}')
    return code
