"""B200-native hybrid mixer-layer forward (attention ∥ Mamba-2), a drop-in for the layer harness of
anuragdutt/multi_modal_parallelism: same layer config, sharding-recipe and layer API, with every hot op a
hand-written sm_100a kernel behind the C-ABI library ``libmmp_b200.so``."""
__version__ = "0.1.0"
