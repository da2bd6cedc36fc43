"""qi_b200 — B200-native (sm_100a) kernels for hongzicong/qi's quantized
nn.Linear path: INT8 W8A8, FP8-E4M3 W8A8, W4A16 INT4 and NVFP4 W4A4 GEMMs
behind the reference's WeightOnlyLinear / get_backend / quantized-checkpoint
API.  The kernels live in ``libqi_b200.so`` (C ABI: include/qi_b200.h)."""

__version__ = "0.1.0"
