"""d1 -- B200-native batched D:1 environment step feeding PPO.

Python side of libd1.so (built in-tree from ../csrc for sm_100a). The modules
mirror the reference's own Python entry points:

* d1.learn_env  -- `Env` of gpu-d1/scripts/learn_env.py (reference-compatible task)
* d1.spec_env   -- the BASELINE task (generated maps, 12 semantic actions)
* d1.ppo        -- rollout / GAE / PPO update of gpu-d1/scripts/run_ring_ablations.py

There is no CPU fallback: importing a module that needs the library raises if
libd1.so is missing, and every call checks the library's error code.
"""
