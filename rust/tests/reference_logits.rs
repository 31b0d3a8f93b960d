// The reference's own golden tests (src/model.rs:791-858 and :860-932) run
// against the B200 library: the 18-token prefill logits and the following
// step's logits of the real Pebble-25M checkpoint within 1e-4 max-abs, and
// their argmaxes 199 and 490.  Like the reference, the test passes without
// doing anything when the checkpoint or the golden files are absent
// (KRIKIL_PEBBLE_WEIGHTS names the checkpoint; KRIKIL_GOLDEN_DIR the directory
// holding test_reference_logits.json and test_reference_step_logits.json,
// default tests/golden of this repository).
use krikil_b200::{PebbleModel, PebbleState};
use std::path::PathBuf;

fn golden(name: &str) -> Option<(Vec<u32>, Vec<f32>, Option<u32>)> {
    let dir = std::env::var("KRIKIL_GOLDEN_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env!("CARGO_MANIFEST_DIR")).join("../tests/golden")
    });
    let text = std::fs::read_to_string(dir.join(name)).ok()?;
    // minimal reader for {"tokens":[...],"logits":[...],"step_token":n}
    let grab = |key: &str| -> Option<String> {
        let i = text.find(&format!("\"{}\"", key))?;
        let rest = &text[i..];
        let a = rest.find('[')?;
        let b = rest.find(']')?;
        Some(rest[a + 1..b].to_string())
    };
    let tokens = grab("tokens")?.split(',').filter_map(|t| t.trim().parse().ok()).collect();
    let logits = grab("logits")?.split(',').filter_map(|t| t.trim().parse().ok()).collect();
    let step = text.find("\"step_token\"").and_then(|i| {
        let rest = &text[i + 12..];
        let digits: String = rest.chars().skip_while(|c| !c.is_ascii_digit()).take_while(|c| c.is_ascii_digit()).collect();
        digits.parse().ok()
    });
    Some((tokens, logits, step))
}

fn argmax(v: &[f32]) -> usize {
    let mut best = 0;
    for (i, &x) in v.iter().enumerate() {
        if x > v[best] {
            best = i;
        }
    }
    best
}

#[test]
fn prefill_and_step_logits_match_the_reference() {
    let Ok(weights) = std::env::var("KRIKIL_PEBBLE_WEIGHTS") else { return };
    let (Some((tokens, want, _)), Some((_, want_step, step_token))) =
        (golden("reference_prefill_logits.json"), golden("reference_step_logits.json"))
    else {
        return;
    };
    let model = PebbleModel::load_safetensors(&weights).expect("load");
    let mut state = PebbleState::new(&model.config, 2048);
    let got = model.forward_prefill(&tokens, &mut state).expect("prefill");
    let err = got.iter().zip(&want).map(|(a, b)| (a - b).abs()).fold(0.0f32, f32::max);
    assert!(err < 1e-4, "prefill max abs diff {}", err);
    assert_eq!(argmax(&got), 199);
    let got = model.forward_step(step_token.unwrap_or(199), &mut state).expect("step");
    let err = got.iter().zip(&want_step).map(|(a, b)| (a - b).abs()).fold(0.0f32, f32::max);
    assert!(err < 1e-4, "step max abs diff {}", err);
    assert_eq!(argmax(&got), 490);
    assert_eq!(state.current_pos, tokens.len() + 1);
}

#[test]
fn errors_match_the_reference() {
    let Ok(weights) = std::env::var("KRIKIL_PEBBLE_WEIGHTS") else { return };
    let model = PebbleModel::load_safetensors(&weights).expect("load");
    let mut state = PebbleState::new(&model.config, 8);
    assert_eq!(model.forward_prefill(&[], &mut state).unwrap_err().to_string(), "Cannot prefill empty sequence");
    assert_eq!(model.forward_prefill(&[1, 2048], &mut state).unwrap_err().to_string(),
               "Token ID 2048 exceeds vocab size 2048");
    assert_eq!(model.forward_prefill(&[1; 9], &mut state).unwrap_err().to_string(),
               "Sequence length 9 exceeds context limit 8");
    model.forward_prefill(&[1; 8], &mut state).unwrap();
    assert_eq!(model.forward_step(3, &mut state).unwrap_err().to_string(), "Context limit 8 reached");
    assert_eq!(state.current_pos, 8);
}
