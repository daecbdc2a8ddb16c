"""Log-mel features on the GPU (src/audio.rs:192-237) against the host restatement (MelBank::features) on the same
clips: the DFT keeps the host's f64 summation order and roundings, so the power spectra are equal and the features
agree to within one f32 rounding of log10 (which the host takes in f32, the GPU in f64 and rounds)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_SAMPLES = 480000


def _batch(torch, clips):
    audio = np.zeros((len(clips), N_SAMPLES), np.float32)
    for i, c in enumerate(clips):
        audio[i, :min(len(c), N_SAMPLES)] = c[:N_SAMPLES]
    lens = np.array([min(len(c), N_SAMPLES) for c in clips], np.int32)
    return torch.from_numpy(audio).cuda(), torch.from_numpy(lens).cuda()


@pytest.mark.parametrize("n_mels,lengths", [
    (128, [N_SAMPLES, 100000, 4000]),
    (80, [N_SAMPLES - 1, 161, 1, 0]),
    (128, [N_SAMPLES + 12345, 200, 400]),
])
def test_log_mel_gpu_matches_the_host(cuda, n_mels, lengths):
    import mimizuku_b200 as m
    torch = cuda
    clips = [m.synth_clip(7 * i + 3, n) if n > 0 else np.zeros(0, np.float32) for i, n in enumerate(lengths)]
    want, frames = m.log_mel_batch(clips, n_mels)
    audio, lens = _batch(torch, clips)
    out = torch.full((len(clips), n_mels, 3000), 123.0, dtype=torch.float32, device="cuda")
    m.log_mel_gpu(audio, lens, n_mels, out)
    got = out.cpu().numpy()
    assert m.status()[0] == 0
    assert np.isfinite(got).all()
    # The power spectra and filterbank sums are the host's; log10 is correctly rounded here (f64, then f32) while the
    # host's f32 log10 is off by one unit in ~1 % of the values: one f32 rounding at |log10| <= 10 (9.5e-7) carried
    # through (x + 4) / 4, which can round once more
    diff = np.abs(got - want)
    assert diff.max() <= 4e-7, float(diff.max())
    assert np.mean(got == want) > 0.97, float(np.mean(got == want))
    assert list(frames) == [min((min(n, N_SAMPLES) + 159) // 160, 3000) for n in lengths]


def test_log_mel_gpu_silence_and_repeat(cuda):
    """All-zero audio gives the floor everywhere; two calls give identical results."""
    import mimizuku_b200 as m
    torch = cuda
    clips = [np.zeros(N_SAMPLES, np.float32), m.synth_clip(11)]
    audio, lens = _batch(torch, clips)
    a = torch.empty((2, 128, 3000), dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    work = torch.empty(m.log_mel_gpu_work_bytes(2), dtype=torch.uint8, device="cuda")
    m.log_mel_gpu(audio, lens, 128, a, work=work)
    m.log_mel_gpu(audio, lens, 128, b, work=work)
    assert torch.equal(a, b)
    want, _ = m.log_mel_batch(clips[:1], 128)
    assert np.array_equal(a[0].cpu().numpy(), want[0])


def test_log_mel_gpu_rejects_small_work(cuda):
    import mimizuku_b200 as m
    torch = cuda
    audio, lens = _batch(torch, [np.zeros(10, np.float32)])
    out = torch.empty((1, 80, 3000), dtype=torch.float32, device="cuda")
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        m.log_mel_gpu(audio, lens, 80, out, work=small)
