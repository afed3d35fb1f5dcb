"""On-device EOS tracking of the frame commit (``hm_frame_commit``) against the
reference's host-side EOS scan of ``generate`` (app/engine.py:432-437)."""
import pytest
import torch

from estudiocanciones_b200 import _lib

pytestmark = pytest.mark.gpu

AUDIO_EOS = 8193


def reference_scan(out, n_frames, N, check=25):
    """The reference's loop: every `check` frames (and at the last one) scan out[a:i+2]
    with a = max(1, i+2-check) and keep each take's first frame with an id >= AUDIO_EOS."""
    ends = [None] * N
    for i in range(n_frames):
        if (i + 1) % check == 0 or i == n_frames - 1:
            a = max(1, i + 2 - check)
            eos = (out[a:i + 2] >= AUDIO_EOS).any(-1)
            for c in range(N):
                if ends[c] is None and eos[:, c].any():
                    ends[c] = a + int(eos[:, c].nonzero()[0, 0])
    return ends


def test_frame_commit_tracks_first_eos_like_the_reference_scan():
    from estudiocanciones_b200 import build
    build.build()
    L = _lib.lib()
    dev = "cuda"
    N, ncb, F = 4, 8, 60
    B = 2 * N  # conditional rows [:N], unconditional [N:]
    g = torch.Generator().manual_seed(5)
    toks = torch.randint(0, AUDIO_EOS, (F, B, ncb), generator=g)
    toks[0, 0, 3] = AUDIO_EOS       # frame 0 is never scanned by the reference
    toks[7, 0, 0] = AUDIO_EOS + 2   # take 0 ends at 7 ...
    toks[9, 0, 5] = AUDIO_EOS       # ... not at a later EOS
    toks[30, 1, 7] = AUDIO_EOS      # take 1: last codebook
    toks[10, N + 2, 1] = AUDIO_EOS  # take 2: EOS only in its unconditional row -> never ends
    toks[12, 3, :] = AUDIO_EOS - 1  # id 8192 is audio, not EOS
    toks[59, 3, 4] = AUDIO_EOS + 3  # take 3: the last frame
    tok_out = torch.zeros(B, ncb, dtype=torch.long, device=dev)
    tok_in = torch.zeros_like(tok_out)
    pos = torch.zeros(B, dtype=torch.long, device=dev)
    stream = torch.zeros(F, N, ncb, dtype=torch.long, device=dev)
    frame = torch.zeros(1, dtype=torch.long, device=dev)
    ends = torch.full((N,), -1, dtype=torch.long, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for f in range(F):
        tok_out.copy_(toks[f])
        rc = L.hm_frame_commit(tok_out.data_ptr(), tok_in.data_ptr(), B, ncb, pos.data_ptr(), N, stream.data_ptr(),
                               frame.data_ptr(), F, ends.data_ptr(), AUDIO_EOS, 0, st)
        assert rc == 0
    torch.cuda.synchronize()
    out = stream.cpu()
    assert torch.equal(out, toks[:, :N])
    assert torch.equal(tok_in.cpu(), toks[-1])
    assert int(frame.item()) == F and pos.cpu().tolist() == [F] * B
    want = reference_scan(out, F - 1, N)
    assert want == [7, 30, None, 59]
    assert ends.cpu().tolist() == [-1 if e is None else e for e in want]


def test_frame_commit_without_ends_tracks_nothing():
    L = _lib.lib()
    dev = "cuda"
    B, ncb = 2, 8
    tok_out = torch.full((B, ncb), AUDIO_EOS, dtype=torch.long, device=dev)
    tok_in = torch.zeros_like(tok_out)
    pos = torch.zeros(B, dtype=torch.long, device=dev)
    frame = torch.ones(1, dtype=torch.long, device=dev)
    rc = L.hm_frame_commit(tok_out.data_ptr(), tok_in.data_ptr(), B, ncb, pos.data_ptr(), 1, None, frame.data_ptr(),
                           0, None, AUDIO_EOS, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(tok_in, tok_out) and int(frame.item()) == 2
    # n_keep outside [0, B] is an argument error
    assert L.hm_frame_commit(tok_out.data_ptr(), tok_in.data_ptr(), B, ncb, pos.data_ptr(), B + 1, None,
                             frame.data_ptr(), 0, None, AUDIO_EOS, 0, None) == _lib.HM_EARG
