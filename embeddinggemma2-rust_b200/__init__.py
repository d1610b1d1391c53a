"""B200-native EmbeddingGemma 2 text-backbone and vision-tower forward (sm_100a library + host layer).

The compute path is the C-ABI library built from ``csrc/`` (``_lib/libeg2_b200.so``); this package
holds the host-side mirror of the reference's backend interface over it (``backend``), the model
configuration (``config``), the safetensors checkpoint format (``weights``) and the reference's
parity tolerance profiles (``verify``).
"""
