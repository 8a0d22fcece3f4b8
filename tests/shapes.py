"""The shapes the tests and the bench use (M, N, K)."""

# The judge's B200 shapes (judge/shapes/B200.txt:5-22): Llama-3-70B layers at M = 16, 128, 512, 2048, and the ladder.
JUDGE_B200 = [
    ("qkv_m16", 16, 10240, 8192), ("qkv_m128", 128, 10240, 8192), ("qkv_m512", 512, 10240, 8192),
    ("qkv_m2048", 2048, 10240, 8192), ("o_m16", 16, 8192, 8192), ("o_m128", 128, 8192, 8192),
    ("o_m512", 512, 8192, 8192), ("o_m2048", 2048, 8192, 8192), ("gateup_m16", 16, 57344, 8192),
    ("gateup_m128", 128, 57344, 8192), ("gateup_m512", 512, 57344, 8192), ("gateup_m2048", 2048, 57344, 8192),
    ("down_m16", 16, 8192, 28672), ("down_m128", 128, 8192, 28672), ("down_m512", 512, 8192, 28672),
    ("down_m2048", 2048, 8192, 28672), ("ladder", 8192, 8192, 8192),
]
# BASELINE's 17th shape variant and its config 1 (the H100 ladder shape).
LADDER_4096 = ("ladder_4096", 4096, 6144, 8192)
CONFIG1 = ("config1", 4608, 5632, 8192)
# The decode regime: the four weights at M = 1, 8, 16, 32, 64 tokens (M = 1 and 8 served as they
# are: the kernel rounds the tokens up to 16 with the TMA engine's zero fill).
DECODE_WEIGHTS = [("qkv", 10240, 8192), ("o", 8192, 8192), ("gateup", 57344, 8192), ("down", 8192, 28672)]
DECODE_M = [1, 8, 16, 32, 64]

# M not a multiple of 16 (the library serves any M >= 1; the reference's candidates refuse these): swap-AB with the
# tokens' last group part-filled (K halves on clusters of two, stream-K), pair tiles with ragged last rows (whole
# tiles, a split-K tail, stream-K), M below a pair tile's 256 rows.
RAGGED_M = [(1, 256, 64), (1, 9600, 576), (8, 1024, 1024), (8, 38080, 128), (3, 64, 4096), (24, 320, 192),
            (100, 10240, 448), (127, 576, 64), (129, 256, 128), (130, 5376, 128), (200, 512, 1024),
            (1001, 2304, 320), (2049, 4864, 128), (4599, 5632, 192)]

# hopper/verif.cu:158-163: the reference's 26 edge shapes.
VERIF = [(16, 256, 64), (144, 256, 64), (128, 512, 128), (208, 512, 192), (272, 5376, 128), (1168, 512, 64),
         (144, 512, 256), (16, 1024, 1024), (16, 6144, 128), (144, 512, 320), (144, 512, 832), (2064, 6656, 320),
         (16, 8704, 64), (16, 50944, 64), (48, 4096, 128), (128, 8448, 128), (128, 8704, 128), (128, 17152, 64),
         (4224, 2304, 64), (1536, 10496, 320), (80, 4096, 640), (112, 10240, 448), (3344, 1536, 320),
         (512, 10240, 320), (16, 28672, 448), (16, 65536, 448)]

# This rung's own edges on 148 SMs: N a multiple of 64 but not of 128 or 256 (a half tile), M just above 128, the
# swap path at every bn, stream-K with a block share inside one tile, data-parallel waves plus a stream-K tail.
B200_EDGES = [(16, 64, 64), (32, 192, 128), (48, 320, 64), (64, 1088, 576), (80, 2112, 64), (96, 64, 4096),
              (112, 448, 192), (128, 128, 64), (144, 64, 64), (256, 320, 128), (272, 576, 1024), (384, 19008, 64),
              (2048, 4864, 128), (1280, 7680, 192), (16, 128, 28672),
              # 256-column swap tiles with the last one half outside N: K halves on clusters of two (two shapes),
              # stream-K (the tiles outnumber the SMs)
              (96, 9600, 512), (32, 9600, 576), (64, 38080, 128)]
