"""The console page (plain HTML + a little JavaScript, no external assets)."""
import json


def page_html(cards: dict, api: dict) -> str:
    models = {k: {'name': m['name'], 'options': m['options']} for k, m in cards.items()}
    return f"""<!doctype html><html><head><meta charset="utf-8"><title>xtier_b200 console</title>
<style>body{{font-family:sans-serif;margin:2em;max-width:60em}} pre{{background:#f4f4f4;padding:1em;max-height:25em;
overflow:auto}} select{{margin:.2em}}</style></head><body>
<h1>xtier_b200 console</h1>
<p><select id="model"></select> <span id="opts"></span>
<button onclick="start()">launch</button> <button onclick="stop()">stop</button></p>
<p id="status">...</p><pre id="log"></pre>
<script>
const MODELS = {json.dumps(models)};
const API = {json.dumps(api)};
function renderOpts() {{
  const m = MODELS[document.getElementById('model').value];
  document.getElementById('opts').innerHTML = m.options.map(o =>
    `${{o.label}}: <select id="opt_${{o.key}}">` + o.choices.map(c =>
      `<option value="${{c[0]}}" ${{c[0]===o.default?'selected':''}}>${{c[1]}}</option>`).join('') + '</select>').join(' ');
}}
function values() {{
  const m = MODELS[document.getElementById('model').value]; const v = {{}};
  m.options.forEach(o => v[o.key] = document.getElementById('opt_' + o.key).value); return v;
}}
async function post(path, body) {{
  const r = await fetch('/' + path, {{method: 'POST', headers: {{'Content-Type': 'application/json',
    'X-Xtier-Console': '1'}}, body: JSON.stringify(body)}}); return r.json();
}}
async function start() {{ await post(API.start, {{model: document.getElementById('model').value, values: values()}}); }}
async function stop() {{ await post(API.stop, {{}}); }}
async function poll() {{
  const s = await (await fetch('/' + API.status)).json();
  let line = s.running ?
    `running ${{s.current.model}} (pid ${{s.current.pid}}) ready=${{s.health && s.health.ready}}` : 'idle';
  if (s.running && s.stage && s.stage.phase !== 'ready') line += ` · ${{s.stage.label}} ${{s.stage.percent}} %`;
  if (s.running && s.telemetry) line += ` · ${{s.telemetry.tok_s.toFixed(1)}} tok/s, queue ${{s.telemetry.queue}}`;
  if (!s.running && s.down_reason) line += ` · stopped: ${{s.down_reason}}`;
  if (!s.running && s.result) line += ` · result: ${{JSON.stringify(s.result).slice(0, 400)}}`;
  document.getElementById('status').textContent = line;
  const j = await (await fetch('/' + API.job)).json();
  document.getElementById('log').textContent = (j.log || s.log || []).join('\\n');
}}
const sel = document.getElementById('model');
Object.keys(MODELS).forEach(k => {{ const o = document.createElement('option'); o.value = k;
  o.textContent = MODELS[k].name; sel.appendChild(o); }});
sel.onchange = renderOpts; renderOpts(); poll(); setInterval(poll, 2000);
</script></body></html>"""
