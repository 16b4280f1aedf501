"""PRA-B200: Progressive Retrieval Attention written for B200 (sm_100a) GPUs.

Layer map (bottom to top):

* ``config`` / ``chunking``        -- configuration and token-exact partitioning
* ``core`` / ``refs`` / ``data``   -- reference tables, datasets, tokenizers, collator
* ``memory``                       -- cache data model, lifecycle, routing, gists,
                                      resolver, recursive builder, paged device store
* ``ops``                          -- sm_100a CUDA kernels behind autograd functions
* ``models``                       -- TinyGPT-PRA and the PRA-patched Llama family
* ``parallel``                     -- NCCL bootstrap, peer-memory collectives, DP/TP
* ``runtime``                      -- training engine, checkpoints, logging, metrics
* ``pra_train`` / ``trainer`` / ``eval`` / ``cli`` -- user entry points
"""

__version__ = "0.1.0"
