"""sq325 — B200-native (sm_100a) Mamba-2 8B hot path with FP4-G16 packed weights and the
52-byte SQ3.25 latent recurrent state.

Host API mirroring the reference's (EndlessChasing/mamb2_8B_FP4_Recall_SQ3.25):
  codec       layout_descriptor, allocate_state, validate_state, scan, PackedState,
              decode_state, encode_state_
  fp4         decode_packet, linear, Fp4Tensor
  checkpoint  load_packed_model, verify_checkpoint, read_state_config (packed on-disk format)
  model       Mamba2FP4Model, synthetic_model, MODEL_CONFIG
  state       PredictorState (reset / backbone / score / greedy)
  resurface   read_fp16, install_fp16
  scoring     ppl_windows, evaluate_ppl, generate
  recall      synthetic_mk_cases, evaluate_mk (the public MK recall protocol)
  state_codec the FP16-state control scan (mode 's16' of mamba2_recall/state_codec.py)
All compute runs in libsq325.so (include/sq325.h); there is no CPU or Triton path.
"""
from . import _lib, checkpoint, codec, fp4, model, recall, resurface, scoring, state, state_codec  # noqa: F401
from .checkpoint import load_packed_model, read_state_config, verify_checkpoint  # noqa: F401
from .codec import LAYOUTS, PackedState, allocate_state, layout_descriptor, scan, validate_state  # noqa: F401
from .model import MODEL_CONFIG, Mamba2FP4Model, synthetic_model  # noqa: F401
from .resurface import install_fp16, read_fp16  # noqa: F401
from .recall import evaluate_mk, synthetic_mk_cases  # noqa: F401
from .scoring import evaluate_ppl, generate, ppl_windows  # noqa: F401
from .state import PredictorState  # noqa: F401
