"""CPU oracle of the sparse-pooling hot path — TEST INFRASTRUCTURE, NOT THE PRODUCT.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker or the timed CPU baseline.
The product (``granulelayer_b200``) never imports it.
"""
