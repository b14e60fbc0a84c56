"""shellsmith_b200: B200 (sm_100a) rollout-cache path of shellsmith's studio_compute.

Device work goes through the C ABI in libshellcache.so (include/shellcache.h):
  numerics   gated_delta_token / gdn_decode   GDN one-token state update
  paged      kv_append / paged_decode_attention / attention_combine
The host side (block manager, scheduler, engine) lives beside them.
"""

__version__ = "0.1.0"
