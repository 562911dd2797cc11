"""The library's soft actor-critic kernels (no reference counterpart), restated in the oracle:
known answers and a finite-difference check of the policy gradient against the objective it
differentiates, J = min(q1, q2) - alpha log pi, for critics linear in the action."""
import numpy as np

from oracle import kernels as K

F32 = np.float32


def test_policy_known_answers():
    A = 3
    out = np.array([0, 0, 0, 0, 0, 0, 0.5, -1.0, 2.0, np.log(2.0), -30.0, 5.0], F32)  # (mu, log_std) x 2
    eps = np.array([0, 0, 0, 1.0, 0.5, -2.0], F32)
    act, lp = np.zeros(2 * A, F32), np.zeros(2, F32)
    K.SACGaussianPolicy(out, eps, act, lp, A, gsize=(2,))
    assert np.all(act[:3] == 0)
    np.testing.assert_allclose(lp[0], 3 * (-0.5 * np.log(2 * np.pi) - np.log(1 + 1e-6)), rtol=1e-6)
    ls = np.array([np.log(2.0), -20.0, 2.0])  # log_std clamped to [-20, 2]
    u = np.array([0.5, -1.0, 2.0]) + np.exp(ls) * eps[3:]
    a = np.tanh(u)
    np.testing.assert_allclose(act[3:], a, rtol=1e-6)
    ref = np.sum(-0.5 * eps[3:].astype(np.float64) ** 2 - ls - 0.5 * np.log(2 * np.pi) - np.log(1 - a * a + 1e-6))
    np.testing.assert_allclose(lp[1], ref, rtol=1e-5)


def test_target_value_known_answers():
    q1 = np.array([1.0, -2.0, 3.0], F32)
    q2 = np.array([2.0, -3.0, 3.0], F32)
    r = np.array([0.5, 1.0, -1.0], F32)
    done = np.array([0.0, 0.0, 1.0], F32)
    lp = np.array([-1.0, 2.0, 7.0], F32)
    y = np.zeros(3, F32)
    K.SACTargetValue(q1, q2, r, done, lp, y, 0.99, 0.2, gsize=(3,))
    np.testing.assert_allclose(y, [0.5 + 0.99 * (1.0 + 0.2), 1.0 + 0.99 * (-3.0 - 0.4), -1.0], rtol=1e-6)


def test_policy_gradient_is_the_derivative_of_the_objective():
    rng = np.random.default_rng(3)
    A, n, alpha = 4, 6, 1e-3
    c1 = (rng.standard_normal((n, A)) * 1e-3)  # dq_k/da of critics linear in the action
    c2 = (rng.standard_normal((n, A)) * 1e-3)
    q0 = rng.standard_normal((n, 2))
    out = np.concatenate([rng.standard_normal((n, A)) * 0.5, rng.uniform(-1.5, 0.5, (n, A))], axis=1)
    eps = rng.standard_normal((n, A))

    def objective(o):
        act, lp = np.zeros(n * A, F32), np.zeros(n, F32)
        K.SACGaussianPolicy(o.astype(F32).ravel(), eps.astype(F32).ravel(), act, lp, A, gsize=(n,))
        # evaluated in float64 from the sampled action for a smooth finite difference
        mu, ls = o[:, :A], o[:, A:]
        a = np.tanh(mu + np.exp(ls) * eps)
        logp = np.sum(-0.5 * eps ** 2 - ls - 0.5 * np.log(2 * np.pi) - np.log(1 - a * a + 1e-6), axis=1)
        q1 = q0[:, 0] + np.sum(c1 * a, axis=1)
        q2 = q0[:, 1] + np.sum(c2 * a, axis=1)
        np.testing.assert_allclose(act.reshape(n, A), a, rtol=1e-5, atol=1e-6)
        return np.minimum(q1, q2) - alpha * logp, q1, q2, a

    J, q1, q2, a = objective(out)
    grad = np.zeros(n * 2 * A, F32)
    K.SACPolicyGradient(out.astype(F32).ravel(), eps.astype(F32).ravel(), a.astype(F32).ravel(), q1.astype(F32),
                        q2.astype(F32), c1.astype(F32).ravel(), c2.astype(F32).ravel(), grad, A, alpha, gsize=(n,))
    grad = grad.reshape(n, 2 * A)
    h = 1e-5
    for j in range(2 * A):
        d = np.zeros_like(out)
        d[:, j] = h
        fd = (objective(out + d)[0] - objective(out - d)[0]) / (2 * h)
        assert np.all(np.abs(grad[:, j]) < K.MAX_GRAD)  # inside the clamp: the raw derivative
        np.testing.assert_allclose(grad[:, j], fd, rtol=2e-3, atol=2e-8)
