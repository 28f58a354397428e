"""Small host-side units (CPU): the sampling-parameter words the runner
uploads next to the decode metadata, and the free-block FIFO that prefix
caching can take a block out of."""
import numpy as np


def test_sampling_words_layout():
    from vllm_b200.sampling_params import SamplingParams
    from vllm_b200.src.model_runner import sampling_words
    from vllm_b200.src.request import Request
    greedy = [Request([1, 2], SamplingParams(temperature=0), 7) for _ in range(2)]
    assert sampling_words(greedy) is None               # all greedy: the argmax kernel
    reqs = [Request([1], SamplingParams(temperature=0.5, top_k=20, top_p=0.9, seed=3), 7),
            Request([1], SamplingParams(temperature=0, top_k=0, top_p=1.0, seed=2**33 + 5), 7)]
    reqs[0].sample_stream, reqs[1].sample_stream = 11, 12
    w = sampling_words(reqs)
    n = 2
    assert w.dtype == np.uint32 and w.size == 5 * n
    np.testing.assert_array_equal(w[:n].view(np.float32), np.float32([0.5, 0.0]))
    np.testing.assert_array_equal(w[n:2 * n].view(np.int32), [20, 0])
    np.testing.assert_array_equal(w[2 * n:3 * n].view(np.float32), np.float32([0.9, 1.0]))
    # seed low word and the request's stream id, per row
    np.testing.assert_array_equal(w[3 * n:].reshape(n, 2), [[3, 11], [5, 12]])


def test_free_block_queue_is_the_reference_fifo():
    from collections import deque

    from vllm_b200.src.kv_cache_manager import Block, FreeBlockQueue
    blocks = [Block(i, 0) for i in range(8)]
    q, ref = FreeBlockQueue(blocks), deque(blocks)
    rng = np.random.default_rng(0)
    taken = []
    for _ in range(200):
        if taken and (rng.random() < 0.5 or not len(q)):
            b = taken.pop(int(rng.integers(len(taken))))
            q.append(b)
            ref.append(b)
        else:
            b1, b2 = q.popleft(), ref.popleft()
            assert b1 is b2
            taken.append(b1)
        assert [b.block_id for b in q] == [b.block_id for b in ref]
    # a block can also leave from the middle (a prefix-cache hit)
    mid = list(q)[len(q) // 2]
    q.remove(mid)
    assert mid not in q and len(q) == len(ref) - 1
